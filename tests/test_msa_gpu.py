"""The MSA-stack block on the ``b200`` backend (B200 only).

The outer product mean, the MSA pair-weighted averaging and the MSA transition run the
kernels of ``csrc/msa.cu`` (tcgen05 GEMMs for the contraction over MSA rows, the output
projection, the head-wise averaging and the projections); the pair track runs the Pairformer
kernels. Checked in master precision (bf16 activations) against the CPU oracle
(``oracle/msa.py``, pinned to the reference's own ``EvoformerBlock`` by
``tests/test_oracle_msa.py``) and against the reference's recorded outputs: relative L2
<= 1e-2 per op and per block, on real positions. Benchmark configuration 4's shape (1024 MSA
rows x 512 tokens) runs one block against the oracle.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
import oracle.msa as omsa  # noqa: E402
from foldforge_b200 import _lib  # noqa: E402
from foldforge_b200.engine import backends, policy  # noqa: E402
from foldforge_b200.engine.evoformer import EvoformerBlock  # noqa: E402
from foldforge_b200.engine.serving import report_observations  # noqa: E402
from foldforge_b200.synthetic import evoformer_state, msa_inputs  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 1e-2


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error() == 0


def _block(state, masked_update="compute"):
    block = EvoformerBlock(masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    block = block.cuda().eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(torch.device("cuda"))
    policy.apply_plan(block, plan, torch.device("cuda"))
    return block


def sub(state, prefix):
    return {k[len(prefix) + 1:]: v for k, v in state.items() if k.startswith(prefix + ".")}


@pytest.mark.parametrize("name", ["evo_s6_n20_masked3", "evo_s33_n40_baseline"])
def test_block_matches_the_reference_and_the_oracle(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    state = evoformer_state(torch.Generator().manual_seed(int(rec["wseed"])), scheme=str(rec["scheme"]))
    msa, z, msa_mask, tokens = msa_inputs(int(rec["n_seq"]), int(rec["n"]), int(rec["iseed"]),
                                          masked_suffix=int(rec["masked"]))
    mb, zb = msa.bfloat16(), z.bfloat16()
    block = _block(state)
    pm = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_m, got_z = block(mb.cuda(), zb.cuda(), msa_mask.cuda(), pm.cuda())
    got_m, got_z = got_m.float().cpu(), got_z.float().cpu()
    want_m, want_z = omsa.evoformer_block(mb.float(), zb.float(), msa_mask, tokens, state)
    valid = pm > 0
    assert oracle.rel_l2(got_z, want_z, valid) < TOL
    assert oracle.rel_l2(got_m[:, tokens > 0], want_m[:, tokens > 0]) < TOL
    # the reference ran on the fp32 inputs: bf16 input rounding is inside the same bar
    assert oracle.rel_l2(got_z, torch.from_numpy(rec["out_pair"]), valid) < TOL
    assert oracle.rel_l2(got_m[:, tokens > 0], torch.from_numpy(rec["out_msa"])[:, tokens > 0]) < TOL
    served = {k: v["served_host_calls"] for k, v in report_observations(block)["modules"].items()}
    assert all(v == {"b200": 1} for v in served.values()), served


@pytest.mark.parametrize("n_seq,n,masked,batch", [(64, 72, 5, 2), (130, 33, 0, 1)])
def test_ops_alone_match_the_oracle(n_seq, n, masked, batch):
    state = evoformer_state(torch.Generator().manual_seed(51), scheme="randomise")
    block = _block(state)
    cases = [msa_inputs(n_seq, n, 60 + b, masked_suffix=masked) for b in range(batch)]
    m = torch.stack([c[0] for c in cases]).bfloat16()
    z = torch.stack([c[1] for c in cases]).bfloat16()
    mm = torch.stack([c[2] for c in cases])
    with torch.no_grad():
        opm = block.outer_product_mean(m.cuda(), (mm > 0).cuda()).float().cpu()
        cols = (mm.amax(dim=1) > 0)
        pwa = block.msa_attention1(m.cuda(), z.cuda(), cols.cuda()).float().cpu()
        tr = block.msa_transition(m.cuda()).float().cpu()
    for b in range(batch):
        want = omsa.outer_product_mean(m[b].float(), mm[b], sub(state, "outer_product_mean"))
        assert oracle.rel_l2(opm[b], want) < TOL
        want = omsa.pair_weighted_averaging(m[b].float(), mm[b], z[b].float(), sub(state, "msa_attention1"))
        # the update itself, beyond what the bf16 rounding of the output alone costs
        floor = oracle.rel_l2(want.bfloat16().float() - m[b].float(), want - m[b].float())
        assert oracle.rel_l2(pwa[b] - m[b].float(), want - m[b].float()) < math.hypot(3e-2, floor)
        assert oracle.rel_l2(pwa[b], want) < TOL
        want = oracle.transition(m[b].float(), sub(state, "msa_transition"))
        assert oracle.rel_l2(tr[b], want) < TOL


def test_benchmark_configuration_4_shape_block():
    """One block at BASELINE configuration 4's shape: 1024 MSA rows x 512 tokens, N(0, 0.02) weights."""
    import os

    torch.set_num_threads(os.cpu_count() or 1)
    state = evoformer_state(torch.Generator().manual_seed(0), scheme="baseline")
    msa, z, msa_mask, tokens = msa_inputs(1024, 512, 0, masked_suffix=26)
    mb, zb = msa.bfloat16(), z.bfloat16()
    del msa, z
    block = _block(state)
    pm = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_m, got_z = block(mb.cuda(), zb.cuda(), msa_mask.cuda(), pm.cuda())
    got_m, got_z = got_m.float().cpu(), got_z.float().cpu()
    want_m, want_z = omsa.evoformer_block(mb.float(), zb.float(), msa_mask, tokens, state)
    assert oracle.rel_l2(got_z, want_z, pm > 0) < TOL
    assert oracle.rel_l2(got_m[:, tokens > 0], want_m[:, tokens > 0]) < TOL
