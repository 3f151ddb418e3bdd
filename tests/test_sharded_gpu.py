"""The row-sharded Pairformer block on the b200 shard kernels (B200 only).

Two ranks run the axial-parallel schedule of ``engine/sharded.py``: with two or more GPUs one
GPU per rank over NCCL; with one GPU both ranks share it and exchange host copies over gloo
(the kernels of the two processes never wait on each other). Checked against the CPU oracle
block (master precision, relative L2 1e-2 as the unsharded block test) and against the
unsharded b200 block on the same weights; in "zero" mode masked pairs / tokens are exact.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from foldforge_b200 import _lib  # noqa: E402
from foldforge_b200.engine import backends, graph, policy  # noqa: E402
from foldforge_b200.engine.pairformer import pairformer_block  # noqa: E402
from foldforge_b200.engine.sharded import ShardComm, ShardedPairformerBlock  # noqa: E402
from foldforge_b200.synthetic import block_state, inputs  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _block(state, masked_update):
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    return block.eval()


def _rank(rank: int, world: int, port: int, n: int, masked: int, zero: bool, trimul: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    ngpu = torch.cuda.device_count()
    nccl = ngpu >= world
    dev = torch.device("cuda", rank if nccl else 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl" if nccl else "gloo", rank=rank, world_size=world,
                            device_id=dev if nccl else None)
    comm = ShardComm(trimul=trimul)
    try:
        state = block_state(torch.Generator().manual_seed(31), scheme="randomise")
        z, s, tokens = inputs(n, 4, masked_suffix=masked)
        zb, sb = z.bfloat16(), s.bfloat16()
        r, row0 = comm.rows(n)
        block = _block(state, "zero" if zero else "compute")
        sharded = ShardedPairformerBlock(block, comm, ops="b200", masked_zero=zero)
        with torch.no_grad():
            z_rows, s_out = sharded(zb[row0:row0 + r].to(dev).contiguous(), tokens.to(dev), sb.to(dev))
            z_all = comm.gather_rows(z_rows).float().cpu()
            s_out = s_out.float().cpu()
        assert _lib.device_error() == 0
        want_z, want_s = oracle.pairformer_block(zb.float(), sb.float(), tokens, state)
        pm = (tokens[:, None] * tokens[None, :]) > 0
        if zero:
            assert torch.equal(z_all[~pm], zb.float()[~pm])
            assert torch.equal(s_out[tokens == 0], sb.float()[tokens == 0])
            assert oracle.rel_l2(z_all[pm], want_z[pm]) < 1e-2
            assert oracle.rel_l2(s_out[tokens > 0], want_s[tokens > 0]) < 1e-2
        else:
            assert oracle.rel_l2(z_all, want_z) < 1e-2
            assert oracle.rel_l2(s_out, want_s) < 1e-2
        # the unsharded b200 block on the same weights agrees to bf16 rounding
        if rank == 0:
            one = block.to(dev)
            plan = backends.BackendPlan.make("b200", unsupported="error").resolve(dev)
            policy.apply_plan(torch.nn.ModuleList([one]), plan, dev)
            with torch.no_grad():
                ref_z, ref_s = graph.run_block(one, zb.to(dev), (tokens[:, None] * tokens[None, :]).to(dev),
                                               sb.to(dev), tokens.to(dev))
            assert oracle.rel_l2(z_all, ref_z.float().cpu()) < 1e-2
            assert oracle.rel_l2(s_out, ref_s.float().cpu()) < 1e-2
    finally:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("n,masked,zero,trimul", [(64, 5, False, "auto"), (256, 13, True, "auto"),
                                                  (192, 9, True, "channels")])
def test_two_rank_sharded_block(n, masked, zero, trimul):
    """``trimul="channels"`` forces the channel-sharded TriMul contraction (the default from
    four ranks on) onto the two ranks, when they have a GPU each."""
    mp.spawn(_rank, args=(2, _free_port(), n, masked, zero, trimul), nprocs=2, join=True)


def _exchange_rank(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    peer = ShardComm()
    try:
        ref = ShardComm(peer="off")
        n = 40 * world
        r, row0 = peer.rows(n)
        g = torch.Generator().manual_seed(100 + rank)
        for rep in range(3):  # alternating transpose buffers, interleaved gathers
            x = torch.randn(r, n, 128, generator=g).bfloat16().to(dev)
            small = torch.randn(r, 4, 48, generator=g).bfloat16().to(dev)
            y, y_ref = peer.transpose(x).clone(), ref.transpose(x)
            assert torch.equal(y, y_ref)
            assert torch.equal(peer.gather_rows(small).clone(), ref.gather_rows(small))
            assert torch.equal(peer.transpose(y).clone(), x)
        assert peer._peer is not None  # the peer-memory path ran
        assert _lib.device_error() == 0
    finally:
        peer.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="the peer-memory exchange needs one GPU per rank")
def test_peer_memory_exchanges_match_nccl():
    mp.spawn(_exchange_rank, args=(2, _free_port()), nprocs=2, join=True)
