"""The Pairformer block on the ``b200`` backend (B200 only).

* against the CPU oracle on the same seeded weights and inputs, master precision: every
  output within relative L2 1e-2 ("compute" mode: every position), the update within the
  reference's bf16 tolerance;
* against this package's ``pytorch`` backend under bf16 autocast, the reference's own GPU
  check (``tests/kernels/test_backends_cuda.py:32-65``: relative RMS < 0.03 on pair and
  single), with the observation report showing that ``b200`` served every op;
* a short trunk: drift per block against the fp32 oracle.
"""

from __future__ import annotations

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from foldforge_b200 import _lib  # noqa: E402
from foldforge_b200.engine import backends, graph, policy  # noqa: E402
from foldforge_b200.engine.pairformer import pairformer_block  # noqa: E402
from foldforge_b200.engine.serving import report_observations  # noqa: E402
from foldforge_b200.synthetic import block_state, inputs, trunk_state  # noqa: E402


def rms(a, b):
    a, b = a.float(), b.float()
    return ((a - b).square().mean().sqrt() / b.square().mean().sqrt().clamp_min(1e-6)).item()


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error() == 0


def make_block(state, masked_update="compute"):
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    block = block.cuda().eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(torch.device("cuda"))
    policy.apply_plan(torch.nn.ModuleList([block]), plan, torch.device("cuda"))
    return block


@pytest.mark.parametrize("n,masked", [(24, 3), (130, 11), (64, 0)])
def test_block_matches_oracle(n, masked):
    state = block_state(torch.Generator().manual_seed(21), scheme="randomise")
    block = make_block(state)
    z, s, tokens = inputs(n, 2, masked_suffix=masked)
    zb, sb = z.bfloat16(), s.bfloat16()
    pair_mask = tokens[:, None] * tokens[None, :]
    with torch.no_grad():
        got_pair, got_single = graph.run_block(block, zb.cuda(), pair_mask.cuda(), sb.cuda(), tokens.cuda())
    want_pair, want_single = oracle.pairformer_block(zb.float(), sb.float(), tokens, state)
    got_pair, got_single = got_pair.float().cpu(), got_single.float().cpu()
    assert oracle.rel_l2(got_pair, want_pair) < 1e-2
    assert oracle.rel_l2(got_single, want_single) < 1e-2
    assert oracle.rel_l2(got_pair - zb.float(), want_pair - zb.float()) < 3e-2
    assert oracle.rel_l2(got_single - sb.float(), want_single - sb.float()) < 3e-2
    served = report_observations(block)["modules"]
    assert served and all(v["served_host_calls"] == {"b200": 1} for v in served.values()), served


def test_block_policy_matches_pytorch_backend_under_autocast():
    torch.manual_seed(1)
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, n_head_single=16).cuda().eval()
    with torch.no_grad():
        for p in block.parameters():
            if p.ndim > 1:
                p.normal_(0, 0.05)
    reference = copy.deepcopy(block)
    plan = backends.BackendPlan.make("miniworld").resolve(torch.device("cuda"))
    choices = policy.apply_plan(torch.nn.ModuleList([block]), plan, torch.device("cuda"))
    assert choices and all(c["backend"] == "b200" for c in choices.values())
    pair = torch.randn(1, 128, 128, 128, device="cuda", dtype=torch.bfloat16)
    single = torch.randn(1, 128, 384, device="cuda", dtype=torch.bfloat16)
    mask = torch.ones(1, 128, device="cuda", dtype=torch.bool)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        expected = reference(pair.clone(), mask, single.clone())
        actual = block(pair.clone(), mask, single.clone())
    assert rms(actual[0], expected[0]) < 0.03
    assert rms(actual[1], expected[1]) < 0.03
    ran = {k: v["served_host_calls"] for k, v in report_observations(block)["modules"].items()}
    assert all(calls == {"b200": 1} for calls in ran.values()), ran


def test_masked_zero_block_leaves_padding_exactly():
    state = block_state(torch.Generator().manual_seed(22), scheme="randomise")
    block = make_block(state, masked_update="zero")
    z, s, tokens = inputs(100, 3, masked_suffix=7)
    zb, sb = z.bfloat16().cuda(), s.bfloat16().cuda()
    pair_mask = (tokens[:, None] * tokens[None, :]).cuda()
    with torch.no_grad():
        got_pair, got_single = graph.run_block(block, zb, pair_mask, sb, tokens.cuda())
    assert torch.equal(got_pair[pair_mask == 0], zb[pair_mask == 0])
    assert torch.equal(got_single[tokens.cuda() == 0], sb[tokens.cuda() == 0])
    want_pair, want_single = oracle.pairformer_block(zb.float().cpu(), sb.float().cpu(), tokens, state)
    valid = pair_mask.cpu() > 0
    assert oracle.rel_l2(got_pair.float().cpu()[valid], want_pair[valid]) < 1e-2
    assert oracle.rel_l2(got_single.float().cpu()[tokens > 0], want_single[tokens > 0]) < 1e-2


def test_trunk_drift_stays_within_tolerance():
    """Four blocks of the benchmark's weight scheme: master-mode drift per block against fp32."""
    states = trunk_state(4, seed=0)
    blocks = [make_block(st) for st in states]
    z, s, tokens = inputs(96, 0, masked_suffix=5)
    zc, sc = z.bfloat16().cuda(), s.bfloat16().cuda()
    zo, so = z.bfloat16().float(), s.bfloat16().float()
    mask = (tokens > 0)[None].cuda()
    for st, block in zip(states, blocks):
        with torch.no_grad():
            zc, sc = block(zc[None] if zc.dim() == 3 else zc, mask, sc[None] if sc.dim() == 2 else sc)
        zo, so = oracle.pairformer_block(zo, so, tokens, st)
        assert oracle.rel_l2(zc[0].float().cpu(), zo) < 1e-2
        assert oracle.rel_l2(sc[0].float().cpu(), so) < 1e-2
