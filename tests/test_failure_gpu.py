"""Bounded waits run out without faulting the GPU (B200 only, one GPU).

The peer-memory exchanges end with ``ffb_shard_wait_p2p``: the stream waits until every
rank has published the current epoch in this rank's flag array. Here nothing ever publishes
it (a zeroed flag array whose epoch is 1, on one process), so the wait must give up after
its limit, record code 106 in the device error word and let the stream go on: the call
returns, ``ffb_device_error`` reports 106 (and clears it), and the next kernel call on the
same context works.
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

from foldforge_b200 import _lib, kernels  # noqa: E402

TIMEOUT_PEER = 106


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_shard_wait_on_a_flag_nobody_sets_times_out_and_the_context_survives():
    lib = _lib.load()
    assert _lib.device_error() == 0
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")          # slots of P = 2 ranks, never written
    sync = torch.tensor([0, 1], dtype=torch.int32, device="cuda")     # arrival counter, epoch 1
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    start = time.monotonic()
    status = lib.ffb_shard_wait_p2p(_p(flags), _p(sync), 2, 50_000, stream)  # 50 ms limit
    assert status == 0, lib.ffb_last_error()
    assert _lib.device_error() == TIMEOUT_PEER
    elapsed = time.monotonic() - start
    assert 0.04 < elapsed < 5.0, elapsed
    assert _lib.device_error() == 0  # read and cleared
    # the context is usable: a LayerNorm afterwards is correct
    x = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    y = kernels.layer_norm(x, torch.ones(128, device="cuda"), torch.zeros(128, device="cuda"))
    want = torch.nn.functional.layer_norm(x.float(), (128,)).bfloat16()
    torch.testing.assert_close(y.float(), want.float(), rtol=2e-2, atol=2e-2)
    assert _lib.device_error() == 0


def test_shard_wait_returns_at_once_when_every_slot_has_the_epoch():
    lib = _lib.load()
    flags = torch.tensor([1, 1, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device="cuda")
    sync = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    start = time.monotonic()
    assert lib.ffb_shard_wait_p2p(_p(flags), _p(sync), 2, 10_000_000, stream) == 0
    assert _lib.device_error() == 0
    assert time.monotonic() - start < 1.0
