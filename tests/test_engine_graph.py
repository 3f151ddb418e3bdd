"""The engine classes: schema, precision, and the ``pytorch`` backend against the oracle.

Mirrors the reference's ``tests/kernels/test_engine_factories.py`` (fp32 parameters, master
flags) and ``tests/models/test_engine_graph.py:127-148`` (engine ``pytorch`` backend equals
the dense reference block on real positions, fp32, rtol = atol = 1e-4), through FoldForge's
own ``run_block`` layout.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from foldforge_b200.engine import factories, graph
from foldforge_b200.engine.modules import MasterWeights, PairformerBlock, Transition
from foldforge_b200.engine.pairformer import pairformer_block
from foldforge_b200.synthetic import BlockShape, block_schema, block_state, inputs

TOL = {"rtol": 1e-4, "atol": 1e-4}


def test_state_dict_is_the_converter_schema():
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384)
    got = {k: tuple(v.shape) for k, v in block.state_dict().items()}
    assert got == dict(block_schema(BlockShape()))
    assert len(got) == 56


@pytest.mark.parametrize("precision", ["master", "fp32"])
def test_parameters_are_fp32_never_native_bf16(precision):
    module = factories.transition(32, 4, precision=precision)
    assert isinstance(module, Transition)
    assert {p.dtype for p in module.parameters()} == {torch.float32}
    assert module.master_weights is (precision == "master")
    module.to(torch.bfloat16)
    assert module.expand_a.weight.dtype == (torch.float32 if precision == "master" else torch.bfloat16)
    assert module.ln_in.weight.dtype == torch.float32
    with pytest.raises(ValueError, match="precision"):
        factories.finish(Transition(8, 2), "bf16")


def test_master_flag_reaches_every_mixin_below():
    block = pairformer_block(d_pair=32, triangle_model="af3", d_single=64, n_head_single=4)
    mixins = [m for m in block.modules() if isinstance(m, MasterWeights)]
    assert mixins and all(m.master_weights for m in mixins)


def test_model_keys():
    assert factories.model_keys("alphafold3").triangle == "af3"
    with pytest.raises(ValueError, match="no engine selector keys"):
        factories.model_keys("nope")
    with pytest.raises(ValueError):
        factories.triangle_attention(32, 4, starting=True, model="rf3")


def _block(shape: BlockShape, state, masked_update="compute") -> PairformerBlock:
    block = pairformer_block(d_pair=shape.c_z, triangle_model="af3", d_single=shape.c_s,
                             d_hidden_tri_multi=shape.hidden_mul, d_hidden_tri_attention=shape.d_tri,
                             n_head_tri_attention=shape.n_head_pair, n_head_single=shape.n_head_single,
                             precision="fp32", masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    return block.eval()


@pytest.mark.parametrize("n,masked", [(24, 3), (13, 0), (9, 9)])
def test_pytorch_backend_matches_the_oracle(n, masked):
    shape = BlockShape(c_z=32, c_s=64, hidden_mul=32, n_head_pair=4, d_tri=8, n_head_single=4)
    state = block_state(torch.Generator().manual_seed(3), shape, "randomise")
    block = _block(shape, state)
    z, s, tokens = inputs(n, 1, shape.c_z, shape.c_s, masked_suffix=masked)
    pair_mask = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_pair, got_single = graph.run_block(block, z, pair_mask, s.clone(), tokens)
    want_pair, want_single = oracle.pairformer_block(z, s, tokens, state, n_head_pair=4, n_head_single=4)
    torch.testing.assert_close(got_pair, want_pair, **TOL)  # "compute" mode: every position
    torch.testing.assert_close(got_single, want_single, **TOL)


def test_masked_zero_mode_leaves_padding_and_matches_real_positions():
    shape = BlockShape(c_z=32, c_s=64, hidden_mul=32, n_head_pair=4, d_tri=8, n_head_single=4)
    state = block_state(torch.Generator().manual_seed(4), shape, "randomise")
    block = _block(shape, state, masked_update="zero")
    z, s, tokens = inputs(12, 2, shape.c_z, shape.c_s, masked_suffix=4)
    pair_mask = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_pair, got_single = graph.run_block(block, z, pair_mask, s.clone(), tokens)
    assert torch.equal(got_pair[pair_mask == 0], z[pair_mask == 0])
    assert torch.equal(got_single[tokens == 0], s[tokens == 0])


def test_golden_af3_block_through_the_engine_classes():
    rec = dict(np.load("tests/golden/af3_n24_masked3.npz"))
    state = block_state(torch.Generator().manual_seed(int(rec["wseed"])), BlockShape(), str(rec["scheme"]))
    block = _block(BlockShape(), state)
    z, s, _ = inputs(24, int(rec["iseed"]))
    tokens = torch.from_numpy(rec["tokens"])
    pair_mask = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_pair, got_single = graph.run_block(block, z, pair_mask, s.clone(), tokens)
    valid = pair_mask > 0
    torch.testing.assert_close(got_pair[valid], torch.from_numpy(rec["out_pair"])[valid], **TOL)
    torch.testing.assert_close(got_single[tokens > 0], torch.from_numpy(rec["out_single"])[tokens > 0], **TOL)
