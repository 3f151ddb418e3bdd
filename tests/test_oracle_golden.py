"""The CPU oracle reproduces the reference's own legacy block on the golden fixtures.

The fixtures (``tests/golden/*.npz``) were produced by ``tests/golden/make_golden.py``
running FoldForge's released-layout ``PairformerBlock`` (``legacy/pairformer.py:37-229``).
Weights and inputs are re-drawn here from the recorded seeds; their digests must match the
ones recorded next to the reference outputs, so both sides read identical numbers.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from foldforge_b200.synthetic import BlockShape, block_state, inputs

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("evo_", "dit_")))  # Pairformer cases
#: the reference's own fp32 parity tolerance (tests/models/test_engine_graph.py:27)
TOL = {"rtol": 1e-4, "atol": 1e-4}


def _digest(state):
    h = hashlib.sha256()
    for k in sorted(state):
        h.update(k.encode())
        h.update(state[k].contiguous().numpy().tobytes())
    return h.hexdigest()


def load(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    dims = [int(x) for x in rec["shape"]]
    shape = BlockShape(*dims)
    state = block_state(torch.Generator().manual_seed(int(rec["wseed"])), shape, str(rec["scheme"]))
    z, s, _ = inputs(int(rec["n"]), int(rec["iseed"]), shape.c_z, shape.c_s)
    tokens = torch.from_numpy(rec["tokens"])
    return rec, shape, state, z, s, tokens


def sub(state, prefix):
    return {k[len(prefix) + 1 :]: v for k, v in state.items() if k.startswith(prefix + ".")}


@pytest.mark.parametrize("name", CASES)
def test_seeds_reproduce_the_recorded_weights_and_inputs(name):
    rec, _, state, z, s, _ = load(name)
    assert _digest(state) == str(rec["weights_sha256"])
    assert _digest({"z": z, "s": s}) == str(rec["inputs_sha256"])


@pytest.mark.parametrize("name", CASES)
def test_block_matches_reference_everywhere(name):
    rec, shape, state, z, s, tokens = load(name)
    bias = torch.from_numpy(rec["extra_pair_bias"]) if "extra_pair_bias" in rec else None
    pair, single = oracle.pairformer_block(
        z, s, tokens, state, n_head_pair=shape.n_head_pair, n_head_single=shape.n_head_single,
        extra_pair_bias=bias,
    )
    torch.testing.assert_close(single, torch.from_numpy(rec["out_single"]), **TOL)
    if "rows" in rec:
        torch.testing.assert_close(pair[torch.from_numpy(rec["rows"])], torch.from_numpy(rec["out_pair_rows"]), **TOL)
    else:
        torch.testing.assert_close(pair, torch.from_numpy(rec["out_pair"]), **TOL)
    assert abs(pair.double().sum().item() - float(rec["pair_sum"])) <= 1e-4 * max(1.0, abs(float(rec["pair_sumsq"])) ** 0.5)
    assert pair.double().square().sum().item() == pytest.approx(float(rec["pair_sumsq"]), rel=1e-5)
    assert single.double().square().sum().item() == pytest.approx(float(rec["single_sumsq"]), rel=1e-5)


@pytest.mark.parametrize("name", [c for c in CASES if "op.tri_multi_outgoing" in np.load(GOLDEN / f"{c}.npz")])
def test_each_op_matches_reference(name):
    rec, shape, state, z, s, tokens = load(name)
    bias = torch.from_numpy(rec["extra_pair_bias"]) if "extra_pair_bias" in rec else None
    got = {
        "tri_multi_outgoing": oracle.triangle_multiplication(z, tokens, sub(state, "tri_multi_outgoing"), outgoing=True),
        "tri_multi_incoming": oracle.triangle_multiplication(z, tokens, sub(state, "tri_multi_incoming"), outgoing=False),
        "tri_atten_starting": oracle.triangle_attention(z, tokens, sub(state, "tri_atten_starting"), starting=True, n_head=shape.n_head_pair),
        "tri_atten_ending": oracle.triangle_attention(z, tokens, sub(state, "tri_atten_ending"), starting=False, n_head=shape.n_head_pair),
        "transition_pair": oracle.transition(z, sub(state, "transition_pair")),
        "single_transition": oracle.transition(s, sub(state, "single_transition")),
        "single_attention": oracle.attention_pair_bias(s, z, tokens, sub(state, "single_attention"),
                                                       n_head=shape.n_head_single, extra_pair_bias=bias),
    }
    for op, value in got.items():
        torch.testing.assert_close(value, torch.from_numpy(rec[f"op.{op}"]), **TOL, msg=op)


def test_float64_oracle_agrees_with_float32():
    rec, shape, state, z, s, tokens = load("af3_n24_masked3")
    p32, s32 = oracle.pairformer_block(z, s, tokens, state)
    p64, s64 = oracle.pairformer_block(z, s, tokens, state, dtype=torch.float64)
    assert oracle.rel_l2(p32, p64) < 1e-6
    assert oracle.rel_l2(s32, s64) < 1e-6


def test_a_planted_error_is_caught():
    """A wrong oracle (incoming contracted like outgoing) must fail the golden check."""
    rec, shape, state, z, s, tokens = load("small_n13_ragged")
    wrong = oracle.triangle_multiplication(z, tokens, sub(state, "tri_multi_incoming"), outgoing=True)
    assert not torch.allclose(wrong, torch.from_numpy(rec["op.tri_multi_incoming"]), **TOL)
