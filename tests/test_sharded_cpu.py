"""Row-sharded (axial-parallel) Pairformer block on CPU ranks (gloo, world size 2 and 4).

The schedule of ``engine/sharded.py`` with its fp32 torch ops must reproduce the unsharded
oracle block (``oracle.pairformer_block``, the restatement pinned to the reference's own
legacy block) at the engine's fp32 tolerance: this checks the all-to-all transposes, the
row gathers, the left / right swap that turns TriMul incoming into outgoing on z^T and the
untransposed bias of the ending node.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from foldforge_b200.engine.pairformer import pairformer_block
from foldforge_b200.engine.sharded import ShardComm, ShardedPairformerBlock, swapped_trimul_weights
from foldforge_b200.synthetic import BlockShape, block_state, inputs

SHAPE = BlockShape(c_z=32, c_s=64, hidden_mul=32, n_head_pair=4, d_tri=8, n_head_single=4)
TOL = dict(rtol=1e-5, atol=1e-5)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _block(state, masked_update):
    block = pairformer_block(d_pair=SHAPE.c_z, triangle_model="af3", d_single=SHAPE.c_s,
                             d_hidden_tri_multi=SHAPE.hidden_mul, d_hidden_tri_attention=SHAPE.d_tri,
                             n_head_tri_attention=SHAPE.n_head_pair, n_head_single=SHAPE.n_head_single,
                             precision="fp32", masked_update=masked_update)
    block.load_state_dict(state, strict=True)
    return block.eval()


def _rank(rank: int, world: int, port: int, n: int, masked: int, zero: bool) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(2)
        state = block_state(torch.Generator().manual_seed(11), SHAPE, "randomise")
        z, s, tokens = inputs(n, 5, SHAPE.c_z, SHAPE.c_s, masked_suffix=masked)
        comm = ShardComm()
        r, row0 = comm.rows(n)
        sharded = ShardedPairformerBlock(_block(state, "zero" if zero else "compute"), comm, ops="torch",
                                         masked_zero=zero)
        with torch.no_grad():
            z_rows, s_out = sharded(z[row0:row0 + r].clone(), tokens, s.clone())
            z_all = comm.gather_rows(z_rows)
            want_z, want_s = oracle.pairformer_block(z, s, tokens, state, n_head_pair=4, n_head_single=4)
        if zero:
            pm = (tokens[:, None] * tokens[None, :]) > 0
            assert torch.equal(z_all[~pm], z[~pm])
            torch.testing.assert_close(z_all[pm], want_z[pm], **TOL)
            torch.testing.assert_close(s_out[tokens > 0], want_s[tokens > 0], **TOL)
            assert torch.equal(s_out[tokens == 0], s[tokens == 0])
        else:
            torch.testing.assert_close(z_all, want_z, **TOL)
            torch.testing.assert_close(s_out, want_s, **TOL)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,masked,zero", [(2, 12, 3, False), (2, 16, 0, False), (4, 16, 5, False),
                                                 (2, 12, 4, True)])
def test_sharded_block_matches_the_oracle(world, n, masked, zero):
    mp.spawn(_rank, args=(world, _free_port(), n, masked, zero), nprocs=world, join=True)


def _transpose_rank(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, c = 4 * world, 3
        z = torch.arange(n * n * c, dtype=torch.float32).reshape(n, n, c)
        comm = ShardComm()
        r, row0 = comm.rows(n)
        y = comm.transpose(z[row0:row0 + r].contiguous())
        assert torch.equal(y, z.transpose(0, 1)[row0:row0 + r])
        assert torch.equal(comm.transpose(y), z[row0:row0 + r])
        assert torch.equal(comm.gather_rows(z[row0:row0 + r].contiguous()), z)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_all_to_all_transpose_and_row_gather(world):
    mp.spawn(_transpose_rank, args=(world, _free_port()), nprocs=world, join=True)


def test_incoming_is_outgoing_on_the_transpose_with_left_and_right_swapped():
    state = block_state(torch.Generator().manual_seed(12), SHAPE, "randomise")
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in state.items() if k.startswith(pre + ".")}  # noqa: E731
    z, _, tokens = inputs(10, 6, SHAPE.c_z, SHAPE.c_s, masked_suffix=2)
    w = sub("tri_multi_incoming")
    incoming = oracle.triangle_multiplication(z, tokens, w, outgoing=False)
    via_t = oracle.triangle_multiplication(z.transpose(0, 1), tokens, swapped_trimul_weights(w), outgoing=True)
    torch.testing.assert_close(via_t.transpose(0, 1), incoming, **TOL)


def test_rows_refuses_an_uneven_split():
    comm = ShardComm()
    assert comm.rows(12) == (12, 0)
    comm.world = 5
    with pytest.raises(ValueError):
        comm.rows(12)


def test_peer_path_needs_one_host_and_a_device_per_rank():
    from foldforge_b200.engine.sharded import peer_path_allowed

    assert peer_path_allowed([("h", "gpu-0"), ("h", "gpu-1")])
    assert not peer_path_allowed([("h", "gpu-0"), ("h", "gpu-0")])      # two ranks on one GPU
    assert not peer_path_allowed([("h1", "gpu-0"), ("h2", "gpu-1")])    # two hosts: no CUDA IPC
    assert not peer_path_allowed([("h", f"gpu-{i}") for i in range(9)])  # more ranks than the kernels take
    assert not peer_path_allowed([("h", "gpu-0")])


def _identity_rank(rank: int, world: int, port: int, fake: list, expect: bool) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert ShardComm().peer_capable(identity=tuple(fake[rank])) is expect
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fake,expect", [([("h", "gpu-0"), ("h", "gpu-1")], True),
                                         ([("h", "gpu-3"), ("h", "gpu-3")], False),
                                         ([("a", "gpu-0"), ("b", "gpu-1")], False)])
def test_ranks_agree_on_the_exchange_path_from_their_identities(fake, expect):
    """Every rank gathers the (host, device) identities and takes the same decision: a shared
    GPU or a second host sends the exchanges to the NCCL / gloo collectives."""
    mp.spawn(_identity_rank, args=(2, _free_port(), fake, expect), nprocs=2, join=True)


def _leaving_rank(rank: int, world: int, port: int, queue) -> None:
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    comm = ShardComm()
    n = 4 * world
    z = torch.arange(n * n * 3, dtype=torch.float32).reshape(n, n, 3)
    r, row0 = comm.rows(n)
    rows = z[row0:row0 + r].contiguous()
    comm.transpose(rows)  # step 1: every rank takes part
    if rank == world - 1:
        queue.put(("left", rank))
        queue.close()
        queue.join_thread()  # the message is out before the process goes
        os._exit(0)  # leaves between steps, with nothing in flight
    start = time.monotonic()
    try:
        comm.transpose(rows)  # step 2: the peer is gone
    except Exception as exc:  # noqa: BLE001 - any error from the collective is the expected outcome
        queue.put(("error", rank, type(exc).__name__, time.monotonic() - start))
    else:
        queue.put(("completed", rank))
    queue.close()
    queue.join_thread()
    os._exit(0)


def test_a_rank_that_leaves_between_steps_ends_the_next_exchange_with_an_error():
    """A rank exits between two blocks; the other rank's next transpose must end with an error
    within the process group's short timeout instead of waiting for good."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank was still waiting after 120 s"
    results = sorted((queue.get(timeout=5) for _ in range(2)), key=lambda t: t[1])
    assert results[1] == ("left", 1)
    outcome = results[0]
    assert outcome[0] == "error", outcome
    assert outcome[3] < 60.0, outcome
