"""The single transition's no-allocation entry point (B200 only).

``ffb_single_transition_fwd_noalloc`` serves callers that may not allocate device memory
while they run the op (their memory belongs to a pool or arena of their own, or they
allocate only at start-up): its scratch lives in a fixed array inside the library, so the
caller passes inputs, outputs and packed weights only. This checks, through the C ABI,
that calls in a row (of different sizes and masked-position policies, so each later call
runs on what the one before left in the shared array) give the workspace entry point's
results and agree with the CPU oracle, and that a call beyond the array's 1024-token limit
is refused. The file sorts last so that a run which stops at the first failure has run
every other test before it.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from foldforge_b200 import _lib, kernels  # noqa: E402
from foldforge_b200.synthetic import block_state  # noqa: E402

TOL = 1e-2  # the output tolerance of the other GPU tests
MASKED_COMPUTE, MASKED_ZERO = 0, 1


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_noalloc_single_transition_matches_the_workspace_entry_point():
    lib = _lib.load()
    state = block_state(torch.Generator().manual_seed(31), scheme="randomise")
    weights = {k[len("single_transition.") :]: v for k, v in state.items() if k.startswith("single_transition.")}
    packed = kernels.single_transition_prepare(weights, torch.device("cuda"))
    g = torch.Generator().manual_seed(32)
    # calls in a row: the second fills the whole array, the third runs the compute policy
    for b, n, masked in ((2, 300, MASKED_ZERO), (1, 1024, MASKED_ZERO), (3, 200, MASKED_COMPUTE)):
        s = torch.randn(b, n, 384, generator=g).bfloat16().cuda()
        mask = torch.ones(b, n, dtype=torch.bool)
        mask[:, n - 7 :] = False
        mask_u8 = mask.to(torch.uint8).cuda()
        out = torch.empty_like(s)
        status = lib.ffb_single_transition_fwd_noalloc(_p(s), _p(mask_u8), _p(packed), _p(out), b, n, masked,
                                                       _stream())
        assert status == 0, lib.ffb_last_error().decode()
        want = kernels.single_transition(s, mask.cuda(), packed, masked_zero=masked == MASKED_ZERO)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert oracle.rel_l2(out.float().cpu(), want.float().cpu()) < TOL
        expected = oracle.transition(s.float().cpu(), weights)
        keep = mask if masked == MASKED_ZERO else torch.ones_like(mask)
        assert oracle.rel_l2(out.float().cpu()[keep], expected[keep]) < TOL
        if masked == MASKED_ZERO:
            assert torch.equal(out[~mask.cuda()], s[~mask.cuda()])


def test_noalloc_refuses_more_tokens_than_its_scratch_holds():
    lib = _lib.load()
    s = torch.zeros(1, 1025, 384, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(s)
    packed = torch.zeros(int(lib.ffb_single_transition_packed_bytes()), dtype=torch.uint8, device="cuda")
    status = lib.ffb_single_transition_fwd_noalloc(_p(s), None, _p(packed), _p(out), 1, 1025, 0, _stream())
    assert status == 2
    assert b"1024" in lib.ffb_last_error()
