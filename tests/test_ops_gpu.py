"""Each pair-stack op on the B200 against the CPU oracle (same seeded weights and inputs).

Master precision (fp32 weights, bf16 activations): every op's OUTPUT must be within
relative L2 1e-2 of the fp32 oracle, on every position (the masked ones included) in
"compute" mode. Its UPDATE (output - input) is held to the reference's own bf16 tolerance,
a relative RMS of 0.03 (tests/kernels/test_backends_cuda.py:58-59); the update is measured
through the bf16-rounded output, whose rounding alone is ~2e-3 rms at |z| ~ 1.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from foldforge_b200 import _lib, kernels  # noqa: E402
from foldforge_b200.synthetic import block_state  # noqa: E402

OUT_TOL = 1e-2
DELTA_TOL = 3e-2


def sub(state, prefix):
    return {k[len(prefix) + 1 :]: v for k, v in state.items() if k.startswith(prefix + ".")}


@pytest.fixture(scope="module")
def weights():
    return block_state(torch.Generator().manual_seed(11), scheme="randomise")


def pair_inputs(b, n, masked, seed=0):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(b, n, n, 128, generator=g).bfloat16()
    tokens = torch.ones(b, n)
    for i in range(b):
        if masked:
            tokens[i, n - masked - i :] = 0
    return z, tokens


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error() == 0


CASES = [(1, 24, 3), (1, 130, 10), (2, 64, 5), (1, 256, 13), (1, 1, 0)]


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("b,n,masked", CASES)
def test_trimul_matches_oracle(weights, outgoing, b, n, masked):
    name = "tri_multi_outgoing" if outgoing else "tri_multi_incoming"
    p = sub(weights, name)
    z, tokens = pair_inputs(b, n, masked)
    packed = kernels.trimul_prepare(p, torch.device("cuda"))
    got = kernels.trimul(z.cuda(), tokens.cuda() > 0, packed, outgoing=outgoing, masked_zero=False).float().cpu()
    for i in range(b):
        want = oracle.triangle_multiplication(z[i].float(), tokens[i], p, outgoing=outgoing)
        assert oracle.rel_l2(got[i], want) < OUT_TOL
        assert oracle.rel_l2(got[i] - z[i].float(), want - z[i].float()) < DELTA_TOL


@pytest.mark.parametrize("outgoing", [True, False])
def test_trimul_masked_zero_leaves_padding_untouched(weights, outgoing):
    p = sub(weights, "tri_multi_outgoing" if outgoing else "tri_multi_incoming")
    z, tokens = pair_inputs(1, 150, 20, seed=3)
    packed = kernels.trimul_prepare(p, torch.device("cuda"))
    got = kernels.trimul(z.cuda(), tokens.cuda() > 0, packed, outgoing=outgoing, masked_zero=True).cpu()
    pm = (tokens[0][:, None] * tokens[0][None, :]) > 0
    assert torch.equal(got[0][~pm], z[0][~pm])
    want = oracle.triangle_multiplication(z[0].float(), tokens[0], p, outgoing=outgoing)
    assert oracle.rel_l2(got[0].float()[pm] - z[0].float()[pm], want[pm] - z[0].float()[pm]) < DELTA_TOL


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("b,n,masked", CASES + [(1, 200, 0), (1, 384, 20)])
def test_triattn_matches_oracle(weights, starting, b, n, masked):
    """N = 384: the attention's 256-query units alternate between two query groups and one
    (the second group of the last unit holds no query), which keeps both kinds of step in
    one launch."""
    p = sub(weights, "tri_atten_starting" if starting else "tri_atten_ending")
    z, tokens = pair_inputs(b, n, masked, seed=5)
    packed = kernels.triattn_prepare(p, torch.device("cuda"))
    got = kernels.triattn(z.cuda(), tokens.cuda() > 0, packed, starting=starting, masked_zero=False).float().cpu()
    for i in range(b):
        want = oracle.triangle_attention(z[i].float(), tokens[i], p, starting=starting)
        assert oracle.rel_l2(got[i], want) < OUT_TOL
        assert oracle.rel_l2(got[i] - z[i].float(), want - z[i].float()) < DELTA_TOL


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("n", [640, 800])
def test_trimul_at_lengths_that_leave_a_partial_output_tile(weights, outgoing, n):
    """N not a multiple of the contraction's 256-column tile, with two full 64-column chunks
    before the tile's edge (the weak-scaling lengths of 2 and 4 GPUs). Every column of U must
    be right: no output column may be worse than the bf16 floor of the whole (a staging
    buffer overwritten before its store had read it once corrupted columns 576-583 at 640)."""
    p = sub(weights, "tri_multi_outgoing" if outgoing else "tri_multi_incoming")
    z, tokens = pair_inputs(1, n, 17, seed=12)
    packed = kernels.trimul_prepare(p, torch.device("cuda"))
    got = kernels.trimul(z.cuda(), tokens.cuda() > 0, packed, outgoing=outgoing, masked_zero=False).float().cpu()
    want = oracle.triangle_multiplication(z[0].float(), tokens[0], p, outgoing=outgoing)
    d, u = got[0] - want, want - z[0].float()
    assert oracle.rel_l2(got[0] - z[0].float(), u) < DELTA_TOL
    real = tokens[0] > 0  # padded rows / columns carry near-zero updates: their relative error is noise
    d, u = d[real][:, real], u[real][:, real]
    col = d.pow(2).sum((0, 2)).sqrt() / u.pow(2).sum((0, 2)).sqrt()
    row = d.pow(2).sum((1, 2)).sqrt() / u.pow(2).sum((1, 2)).sqrt()
    assert col.max() < 2 * DELTA_TOL and row.max() < 2 * DELTA_TOL, (col.argmax(), col.max(), row.max())


@pytest.mark.parametrize("starting", [True, False])
def test_triattn_rescale_for_a_late_dominant_key(starting):
    """Weights and inputs under which some queries meet their dominant key only in a late key
    block, so the running maximum is raised and O is rescaled in TMEM mid-row. The rescale must
    wait for exactly the previous step's P V (a barrier phase once taken for an older one let
    it race and corrupted query 5's row at N = 384). Every query row is held to the bf16 floor."""
    w = block_state(torch.Generator().manual_seed(0), scheme="randomise")
    p = sub(w, "tri_atten_starting" if starting else "tri_atten_ending")
    n = 384
    from foldforge_b200.synthetic import inputs

    z, _, tokens = inputs(n, 0, masked_suffix=11)
    zb = z.bfloat16()
    packed = kernels.triattn_prepare(p, torch.device("cuda"))
    mask = (tokens > 0)[None].cuda()
    want = oracle.triangle_attention(zb.float(), tokens, p, starting=starting)
    u = want - zb.float()
    for _ in range(3):  # the race was timing-dependent
        got = kernels.triattn(zb[None].cuda(), mask, packed, starting=starting, masked_zero=False)[0].float().cpu()
        d2, u2 = (got - want).pow(2).sum(-1), u.pow(2).sum(-1)
        axis = 0 if starting else 1  # the problem rows: starting (i = row, j = query), ending (i = query, j = row)
        per_query = (d2.sum(axis) / u2.sum(axis)).sqrt()
        assert oracle.rel_l2(got - zb.float(), u) < DELTA_TOL
        assert per_query.max() < 2 * DELTA_TOL, (per_query.argmax(), per_query.max())


@pytest.mark.parametrize("starting", [True, False])
def test_triattn_fully_masked_rows_average_uniformly(weights, starting):
    """Every token padded: the reference's -1e9 replacement gives uniform weights."""
    p = sub(weights, "tri_atten_starting" if starting else "tri_atten_ending")
    z, tokens = pair_inputs(1, 40, 0, seed=6)
    tokens[:] = 0
    packed = kernels.triattn_prepare(p, torch.device("cuda"))
    got = kernels.triattn(z.cuda(), tokens.cuda() > 0, packed, starting=starting, masked_zero=False).float().cpu()
    want = oracle.triangle_attention(z[0].float(), tokens[0], p, starting=starting)
    assert oracle.rel_l2(got[0] - z[0].float(), want - z[0].float()) < DELTA_TOL
    zero = kernels.triattn(z.cuda(), tokens.cuda() > 0, packed, starting=starting, masked_zero=True).cpu()
    assert torch.equal(zero, z)


@pytest.mark.parametrize("b,n,masked", CASES + [(1, 200, 0)])
def test_pair_transition_matches_oracle(weights, b, n, masked):
    p = sub(weights, "transition_pair")
    z, tokens = pair_inputs(b, n, masked, seed=8)
    packed = kernels.transition_prepare(p, torch.device("cuda"))
    got = kernels.transition(z.cuda(), tokens.cuda() > 0, packed, masked_zero=False).float().cpu()
    for i in range(b):
        want = oracle.transition(z[i].float(), p)
        assert oracle.rel_l2(got[i], want) < OUT_TOL
        assert oracle.rel_l2(got[i] - z[i].float(), want - z[i].float()) < DELTA_TOL
    zero = kernels.transition(z.cuda(), tokens.cuda() > 0, packed, masked_zero=True).cpu()
    for i in range(b):
        pm = (tokens[i][:, None] * tokens[i][None, :]) > 0
        assert torch.equal(zero[i][~pm], z[i][~pm])


def single_inputs(b, n, masked, seed=9):
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(b, n, 384, generator=g).bfloat16()
    z, tokens = pair_inputs(b, n, masked, seed=seed + 1)
    return s, z, tokens


@pytest.mark.parametrize("extra", [False, True])
@pytest.mark.parametrize("b,n,masked", CASES + [(1, 300, 17)])
def test_attention_pair_bias_matches_oracle(weights, extra, b, n, masked):
    p = sub(weights, "single_attention")
    s, z, tokens = single_inputs(b, n, masked)
    bias = torch.randn(n, n, generator=torch.Generator().manual_seed(4)) if extra else None
    packed = kernels.apb_prepare(p, torch.device("cuda"))
    ext = None if bias is None else bias.cuda()[None, None]
    got = kernels.attention_pair_bias(s.cuda(), z.cuda(), tokens.cuda() > 0, packed, extra_pair_bias=ext,
                                      masked_zero=False).float().cpu()
    for i in range(b):
        want = oracle.attention_pair_bias(s[i].float(), z[i].float(), tokens[i], p, extra_pair_bias=bias)
        assert oracle.rel_l2(got[i], want) < OUT_TOL
        assert oracle.rel_l2(got[i] - s[i].float(), want - s[i].float()) < DELTA_TOL


@pytest.mark.parametrize("n,masked,splits", [(160, 9, [(0, 80), (80, 80)]),
                                            (200, 13, [(0, 67), (67, 67), (134, 66)])])
@pytest.mark.parametrize("zero", [False, True])
def test_single_track_by_query_rows_matches_the_whole(weights, n, masked, splits, zero):
    """The row-sharded single track (each rank's queries from its own pair-bias rows,
    ``ffb_apb_shard_single_rows``) reproduces the one-GPU op row for row."""
    import ctypes

    p = sub(weights, "single_attention")
    s, z, tokens = single_inputs(1, n, masked)
    dev = torch.device("cuda")
    packed = kernels.apb_prepare(p, dev)
    mask = (tokens[0] > 0).to(dev)
    whole = kernels.attention_pair_bias(s.to(dev), z.to(dev), mask[None], packed, masked_zero=zero)[0]
    lib = _lib.load()
    ws = torch.empty(int(lib.ffb_apb_single_workspace_bytes(n)), dtype=torch.uint8, device=dev)
    s0, z0, m8 = s[0].to(dev).contiguous(), z[0].to(dev), mask.to(torch.uint8).contiguous()
    parts = []
    for row0, r in splits:
        zr = z0[row0:row0 + r].contiguous()
        pb = torch.empty((r, 16, n), dtype=torch.float32, device=dev)
        _lib.call("ffb_apb_shard_pair_bias", zr.data_ptr(), packed.data_ptr(), pb.data_ptr(), r, n, 0)
        rows = torch.empty((r, 384), dtype=torch.bfloat16, device=dev)
        _lib.call("ffb_apb_shard_single_rows", s0.data_ptr(), m8.data_ptr(), packed.data_ptr(), pb.data_ptr(),
                  ctypes.c_float(0.0), rows.data_ptr(), ws.data_ptr(), ctypes.c_size_t(ws.numel()), n, row0, r,
                  1 if zero else 0, 0)
        parts.append(rows)
    got = torch.cat(parts)
    torch.cuda.synchronize()
    assert torch.equal(got, whole)


@pytest.mark.parametrize("b,n,masked", CASES)
def test_single_transition_matches_oracle(weights, b, n, masked):
    p = sub(weights, "single_transition")
    s, _, tokens = single_inputs(b, n, masked, seed=12)
    packed = kernels.single_transition_prepare(p, torch.device("cuda"))
    got = kernels.single_transition(s.cuda(), tokens.cuda() > 0, packed, masked_zero=False).float().cpu()
    for i in range(b):
        want = oracle.transition(s[i].float(), p)
        assert oracle.rel_l2(got[i], want) < OUT_TOL
        assert oracle.rel_l2(got[i] - s[i].float(), want - s[i].float()) < DELTA_TOL
    zero = kernels.single_transition(s.cuda(), tokens.cuda() > 0, packed, masked_zero=True).cpu()
    for i in range(b):
        assert torch.equal(zero[i][tokens[i] == 0], s[i][tokens[i] == 0])
