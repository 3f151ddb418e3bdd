"""The fp32 precision and the any-width path on the ``b200`` backend (B200 only).

fp32 activations (FoldForge's "fp32" precision) and widths the tcgen05 kernels are not built
for run the FP32 SIMT kernels of ``csrc/generic.cu``. The north star's fp32 bar is relative
L2 <= 1e-5 against the reference; here the b200 block in fp32 is held to that against the
reference's own outputs recorded in ``tests/golden/af3_n128_config1.npz`` (benchmark
configuration 1: N = 128, AF3 widths, N(0, 0.02) weights) and against the CPU oracle on
every golden case (ragged masks, interior padding, an extra pair bias, every token padded,
one token). The template stack's width (c_z = 64, hidden 64, 4 x 16 heads) runs the same
kernels in bf16 and fp32.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from foldforge_b200 import _lib  # noqa: E402
from foldforge_b200.engine import backends, policy  # noqa: E402
from foldforge_b200.engine.pairformer import pairformer_block  # noqa: E402
from foldforge_b200.engine.serving import report_observations  # noqa: E402
from foldforge_b200.synthetic import BlockShape, block_state, inputs  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
FP32_TOL = 1e-5


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error() == 0


def _block(shape: BlockShape, state, precision: str, masked_update: str = "compute"):
    block = pairformer_block(d_pair=shape.c_z, triangle_model="af3", d_single=shape.c_s,
                             d_hidden_tri_multi=shape.hidden_mul, d_hidden_tri_attention=shape.d_tri,
                             n_head_tri_attention=shape.n_head_pair, n_head_single=shape.n_head_single,
                             pair_transition_n=shape.n_pair, single_transition_n=shape.n_single,
                             precision=precision, masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    block = block.cuda().eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(torch.device("cuda"))
    policy.apply_plan(torch.nn.ModuleList([block]), plan, torch.device("cuda"))
    return block


def _golden(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    shape = BlockShape(*[int(x) for x in rec["shape"]])
    state = block_state(torch.Generator().manual_seed(int(rec["wseed"])), shape, str(rec["scheme"]))
    z, s, _ = inputs(int(rec["n"]), int(rec["iseed"]), shape.c_z, shape.c_s)
    return rec, shape, state, z, s, torch.from_numpy(rec["tokens"])


def _run(block, z, s, tokens, extra=None):
    key = (tokens > 0)[None].cuda()
    with torch.no_grad():
        if extra is None:
            pair, single = block(z[None].cuda(), key, s[None].cuda())
        else:
            pair, single = block(z[None].cuda(), key, s[None].cuda(), extra[None, None].cuda())
    return pair[0].cpu(), single[0].cpu()


def test_fp32_block_matches_the_reference_at_benchmark_configuration_1():
    rec, shape, state, z, s, tokens = _golden("af3_n128_config1")
    block = _block(shape, state, "fp32")
    pair, single = _run(block, z, s, tokens)
    assert pair.dtype == torch.float32
    rows = torch.from_numpy(rec["rows"])
    want_rows = torch.from_numpy(rec["out_pair_rows"])
    want_single = torch.from_numpy(rec["out_single"])
    assert oracle.rel_l2(pair[rows], want_rows) <= FP32_TOL
    assert oracle.rel_l2(single, want_single) <= FP32_TOL
    # the whole pair against the recorded checksums of the reference's output
    assert abs(pair.double().sum().item() - float(rec["pair_sum"])) <= 1e-5 * float(rec["pair_sumsq"])
    assert abs(pair.double().square().sum().item() / float(rec["pair_sumsq"]) - 1) <= 2e-5
    served = {k: v["served_host_calls"] for k, v in report_observations(block)["modules"].items()}
    assert all(v == {"b200": 1} for v in served.values()), served


@pytest.mark.parametrize("name", ["af3_n24_masked3", "small_n13_ragged", "small_n5_allmasked", "small_n1"])
def test_fp32_block_matches_the_oracle_on_every_golden_case(name):
    rec, shape, state, z, s, tokens = _golden(name)
    extra = torch.from_numpy(rec["extra_pair_bias"]) if "extra_pair_bias" in rec else None
    block = _block(shape, state, "fp32")
    pair, single = _run(block, z, s, tokens, extra)
    want_pair, want_single = oracle.pairformer_block(z, s, tokens, state, n_head_pair=shape.n_head_pair,
                                                     n_head_single=shape.n_head_single, extra_pair_bias=extra)
    assert oracle.rel_l2(pair, want_pair) <= FP32_TOL
    assert oracle.rel_l2(single, want_single) <= FP32_TOL


@pytest.mark.parametrize("outgoing", [True, False])
def test_fp32_ops_alone_match_the_oracle(outgoing):
    shape = BlockShape()
    state = block_state(torch.Generator().manual_seed(41), shape, "randomise")
    z, s, tokens = inputs(40, 7, masked_suffix=5)
    tokens[11] = 0  # interior padding
    block = _block(shape, state, "fp32", masked_update="compute")
    key = (tokens > 0)[None].cuda()
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in state.items() if k.startswith(pre + ".")}  # noqa: E731
    name = "tri_multi_outgoing" if outgoing else "tri_multi_incoming"
    with torch.no_grad():
        got = getattr(block, name)(z[None].cuda(), key)[0].cpu()
        got_att = block.tri_atten_ending(z[None].cuda(), key)[0].cpu()
    want = oracle.triangle_multiplication(z, tokens, sub(name), outgoing=outgoing)
    want_att = oracle.triangle_attention(z, tokens, sub("tri_atten_ending"), starting=False)
    assert oracle.rel_l2(got, want) <= FP32_TOL
    assert oracle.rel_l2(got_att, want_att) <= FP32_TOL


@pytest.mark.parametrize("precision,tol", [("fp32", FP32_TOL), ("master", 1e-2)])
def test_template_stack_width_runs_on_b200(precision, tol):
    """c_z = 64 (the template stack's pair width), batch 2: the SIMT path in both precisions,
    masked pairs exact in "zero" mode."""
    shape = BlockShape(c_z=64, c_s=0, hidden_mul=64, n_head_pair=4, d_tri=16)
    state = block_state(torch.Generator().manual_seed(42), shape, "randomise", single=False)
    block = pairformer_block(d_pair=64, triangle_model="af3", d_single=0, d_hidden_tri_multi=64,
                             d_hidden_tri_attention=16, n_head_tri_attention=4, precision=precision,
                             masked_update="zero")
    block.load_state_dict(state, strict=True)
    block = block.cuda().eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(torch.device("cuda"))
    policy.apply_plan(torch.nn.ModuleList([block]), plan, torch.device("cuda"))
    dtype = torch.float32 if precision == "fp32" else torch.bfloat16
    g = torch.Generator().manual_seed(43)
    z = torch.randn(2, 30, 30, 64, generator=g).to(dtype)
    tokens = torch.ones(2, 30)
    tokens[0, 26:] = 0
    tokens[1, 3] = 0
    with torch.no_grad():
        got = block(z.cuda(), (tokens > 0).cuda()).cpu()
    for b in range(2):
        want, _ = oracle.pairformer_block(z[b].float(), None, tokens[b], state, n_head_pair=4)
        pm = (tokens[b][:, None] * tokens[b][None, :]) > 0
        assert oracle.rel_l2(got[b].float(), want, pm) <= tol
        assert torch.equal(got[b][~pm], z[b][~pm])
