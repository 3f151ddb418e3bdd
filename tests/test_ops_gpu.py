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
