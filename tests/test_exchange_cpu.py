"""Host-side checks of the row-shard exchange entry points and of the exchange-path choice.

The argument checks of ``ffb_shard_*_p2p`` / ``ffb_p2p_*`` / ``ffb_trimul_channel_contract``
run before any device access, so they are exercised here without a GPU: every malformed
call must come back as FFB_ERR_ARG with a message, never reach a kernel. The path choice of
``ShardComm`` (peer memory only for NCCL groups with a GPU per rank; the channel-sharded
TriMul only on that path) is checked on a single-process group.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from foldforge_b200 import _lib
from foldforge_b200.engine.sharded import ShardComm

ERR_ARG = 1
P = ctypes.c_void_p


def _lib_or_skip():
    if not _lib.LIBRARY.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    return _lib.load()


def _status(lib, name, *args) -> int:
    return getattr(lib, name)(*args)


def _fake(addr: int = 4096) -> ctypes.c_void_p:
    # an aligned, non-null address that the checks must reject before it is ever used
    return P(addr)


@pytest.mark.parametrize("R,N,row0,rank,nranks", [(4, 12, 0, 0, 2),   # N != R P
                                                  (4, 8, 4, 0, 2),    # row0 != rank R
                                                  (4, 8, 0, 2, 2),    # rank out of range
                                                  (4, 36, 0, 0, 9),   # more than 8 ranks
                                                  (0, 0, 0, 0, 2)])   # empty shard
def test_transpose_rejects_inconsistent_shards(R, N, row0, rank, nranks):
    lib = _lib_or_skip()
    st = _status(lib, "ffb_shard_transpose_p2p", _fake(), _fake(), _fake(), _fake(), R, N, row0, rank, nranks, P(0))
    assert st == ERR_ARG
    assert "shard_transpose_p2p" in lib.ffb_last_error().decode()


def test_transpose_rejects_null_and_misaligned_pointers():
    lib = _lib_or_skip()
    assert _status(lib, "ffb_shard_transpose_p2p", P(0), _fake(), _fake(), _fake(), 4, 8, 0, 0, 2, P(0)) == ERR_ARG
    assert _status(lib, "ffb_shard_transpose_p2p", _fake(4098), _fake(), _fake(), _fake(), 4, 8, 0, 0, 2,
                   P(0)) == ERR_ARG


def test_gather_rejects_sizes_that_are_not_whole_16_byte_words():
    lib = _lib_or_skip()
    for nbytes in (0, 24):
        st = _status(lib, "ffb_shard_gather_p2p", _fake(), ctypes.c_size_t(nbytes), _fake(), _fake(), _fake(), 0, 2,
                     P(0))
        assert st == ERR_ARG


@pytest.mark.parametrize("mode,nranks", [(2, 2), (0, 3), (1, 16)])  # unknown mode, 128 % P != 0, P > 8
def test_channel_scatter_rejects_bad_modes_and_rank_counts(mode, nranks):
    lib = _lib_or_skip()
    st = _status(lib, "ffb_shard_rows_p2p", _fake(), mode, 4, 4 * nranks, _fake(), _fake(), _fake(), 0, nranks, P(0))
    assert st == ERR_ARG


def test_wait_rank_count_and_alloc_size_are_checked():
    lib = _lib_or_skip()
    assert _status(lib, "ffb_shard_wait_p2p", _fake(), _fake(), 9, 0, P(0)) == ERR_ARG
    assert _status(lib, "ffb_shard_wait_p2p", P(0), _fake(), 2, 0, P(0)) == ERR_ARG
    # a wait limit above one hour is refused before anything is launched
    assert _status(lib, "ffb_shard_wait_p2p", _fake(), _fake(), 2, 3600 * 10**6 + 1, P(0)) == ERR_ARG
    ptr = P()
    handle = (ctypes.c_uint8 * 64)()
    assert _status(lib, "ffb_p2p_alloc", ctypes.c_size_t(0), ctypes.byref(ptr), handle) == ERR_ARG
    assert _status(lib, "ffb_p2p_open", P(0), ctypes.byref(ptr)) == ERR_ARG


@pytest.mark.parametrize("C,N", [(0, 64), (129, 64), (16, 0)])
def test_channel_contract_rejects_bad_shapes(C, N):
    lib = _lib_or_skip()
    assert _status(lib, "ffb_trimul_channel_contract", _fake(), _fake(), _fake(), C, N, P(0)) == ERR_ARG


def test_handle_size_is_the_cuda_ipc_handle():
    lib = _lib_or_skip()
    assert lib.ffb_p2p_handle_bytes() == 64


def test_single_process_group_uses_local_exchanges_only():
    comm = ShardComm()
    x = torch.arange(4 * 4 * 3, dtype=torch.float32).reshape(4, 4, 3)
    assert comm.world == 1
    assert comm._peer_path(x) is None and not comm.trimul_by_channels(x)
    assert torch.equal(comm.transpose(x), x.transpose(0, 1))
    assert comm.gather_rows(x) is x
    comm.close()  # nothing to unmap
