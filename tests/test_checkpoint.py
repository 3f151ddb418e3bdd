"""Miniworld-format checkpoints (``foldforge_b200.checkpoint``) on the CPU.

The reader applies the checks of FoldForge's ``models/checkpoints/miniworld.py:96-131`` (format
tag, version, family) and takes the pair stack's blocks out of a whole-model state dict by
their AF3 graph prefixes, loading them strictly into this package's classes.
"""

from __future__ import annotations

import pytest
import torch

from foldforge_b200 import checkpoint
from foldforge_b200.synthetic import evoformer_state, inputs, trunk_state


def _model_state(n_trunk=2, n_msa=1):
    state = {"diffusion_head.fourier_embeddings.weight": torch.randn(256),
             "evoformer.single_activations.weight": torch.randn(384, 447)}
    for i, blk in enumerate(trunk_state(n_trunk, seed=3)):
        state.update({f"{checkpoint.TRUNK_PREFIX}.{i}.{k}": v for k, v in blk.items()})
    g = torch.Generator().manual_seed(5)
    for i in range(n_msa):
        state.update({f"{checkpoint.MSA_PREFIX}.{i}.{k}": v for k, v in evoformer_state(g).items()})
    return state


@pytest.fixture
def native(tmp_path):
    state = _model_state()
    path = tmp_path / "af3.miniworld.pt"
    checkpoint.write(path, state, family="alphafold3", source="synthetic")
    return path, state


def test_round_trip_and_tags(native, tmp_path):
    path, state = native
    assert checkpoint.is_native(path) and not checkpoint.is_native(tmp_path / "af3.bin")
    blob = checkpoint.read(path)
    assert blob["family"] == "alphafold3" and blob["version"] == checkpoint.VERSION
    assert set(blob["state_dict"]) == set(state)
    torch.save({"format": "other", "state_dict": {}}, tmp_path / "x.pt")
    with pytest.raises(ValueError, match="not a miniworld-format"):
        checkpoint.read(tmp_path / "x.pt")
    torch.save({"format": "miniworld", "version": 2, "state_dict": {}}, tmp_path / "y.pt")
    with pytest.raises(ValueError, match="version 2"):
        checkpoint.read(tmp_path / "y.pt")
    with pytest.raises(ValueError, match="family"):
        checkpoint.load_trunk(path, family="boltz2", backend="pytorch", dtype=torch.float32, device="cpu")


def test_block_states_by_prefix(native):
    _, state = native
    blocks = checkpoint.block_states(state, checkpoint.TRUNK_PREFIX)
    assert len(blocks) == 2
    for i, blk in enumerate(trunk_state(2, seed=3)):
        assert set(blocks[i]) == set(blk)
        assert all(torch.equal(blocks[i][k], blk[k]) for k in blk)
    assert checkpoint.block_states(state, "evoformer.template_embedding.single_template_embedding") == []
    gap = {k.replace(f"{checkpoint.TRUNK_PREFIX}.1.", f"{checkpoint.TRUNK_PREFIX}.2."): v for k, v in state.items()}
    with pytest.raises(ValueError, match="not 0..1"):
        checkpoint.block_states(gap, checkpoint.TRUNK_PREFIX)


def test_load_trunk_strict_and_equal_to_direct_load(native, tmp_path):
    import foldforge_b200

    path, state = native
    trunk = checkpoint.load_trunk(path, backend="pytorch", dtype=torch.float32, device="cpu")
    direct = foldforge_b200.load(trunk_state(2, seed=3), backend="pytorch", dtype=torch.float32, device="cpu")
    for (ka, va), (kb, vb) in zip(trunk.state_dict().items(), direct.state_dict().items(), strict=True):
        assert ka == kb and torch.equal(va, vb)
    z, s, tok = inputs(12, seed=1, masked_suffix=2)
    with torch.no_grad():
        za, sa = trunk(z[None], (tok > 0)[None], s[None])
        zb, sb = direct(z[None], (tok > 0)[None], s[None])
    assert torch.equal(za, zb) and torch.equal(sa, sb)
    # strictness: a dropped or an extra key of a block is an error
    missing = {k: v for k, v in state.items() if k != f"{checkpoint.TRUNK_PREFIX}.1.transition_pair.squeeze.weight"}
    checkpoint.write(tmp_path / "m.miniworld.pt", missing, family="alphafold3")
    with pytest.raises(RuntimeError, match="Missing key"):
        checkpoint.load_trunk(tmp_path / "m.miniworld.pt", backend="pytorch", dtype=torch.float32, device="cpu")
    extra = dict(state)
    extra[f"{checkpoint.TRUNK_PREFIX}.0.tri_multi_outgoing.spare.weight"] = torch.zeros(1)
    checkpoint.write(tmp_path / "e.miniworld.pt", extra, family="alphafold3")
    with pytest.raises(RuntimeError, match="Unexpected key"):
        checkpoint.load_trunk(tmp_path / "e.miniworld.pt", backend="pytorch", dtype=torch.float32, device="cpu")


def test_load_msa_stack(native):
    path, _ = native
    stack = checkpoint.load_msa_stack(path, backend="pytorch", dtype=torch.float32, device="cpu")
    want = evoformer_state(torch.Generator().manual_seed(5))
    got = stack[0].state_dict()
    assert set(got) == set(want)
    assert all(torch.equal(got[k], want[k]) for k in want)
