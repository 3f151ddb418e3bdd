"""Row-sharded (axial-parallel) Pairformer block over the GPUs of one box.

FoldForge runs the Pairformer on one device; this module adds the pair-axis sharding of the
AF3 trunk across the ranks of one process group (no reference counterpart). Rank r holds the
pair rows ``[r N / P, (r + 1) N / P)`` of ``z [N, N, 128]`` (batch 1); the single track is
replicated. Row-wise ops run on the local rows; the column-wise ops run as their row-wise
counterparts on the transposed pair, reached by an all-to-all:

* TriMul incoming on z = TriMul outgoing on z^T with the left / right projections (and
  their gates) swapped;
* TriAttn ending on z = TriAttn starting on z^T with the UNtransposed pair bias (AF3,
  ``transposed_column_pair_bias=False``), i.e. the transpose of the bias projected from z^T.

Per block: ``TMo (rows) -> A2A -> TMi (z^T rows) -> A2A -> TAs (rows) -> A2A -> TAe (z^T
rows) -> transition (z^T rows) -> A2A -> single track``: four all-to-alls, plus all-gathers
of the TriMul right operand (``[rows][128][Np]`` bf16), the triangle-attention bias rows and
the single-attention pair-bias rows. The b200 ops call the row-sharded C-ABI pieces
(``ffb_*_shard_*``); the torch ops restate the same equations in fp32 for CPU checks of the
schedule (legacy/reference/triangle.py:19-50, legacy/attention.py:108-171,
legacy/reference/transition.py:28-59, legacy/transformer.py:88-133).
"""

from __future__ import annotations

import ctypes
import socket

import torch
import torch.distributed as dist
import torch.nn.functional as F

from foldforge_b200 import _lib

Tensor = torch.Tensor
_LOG2E = 1.4426950408889634


# --------------------------------------------------------------------------- communication
class _CudaArray:
    """A raw device allocation exposed to ``torch.as_tensor`` (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class _PeerBuffer:
    """A device buffer of ``nbytes`` on every rank, each rank's mapped in all the others
    (CUDA IPC through the C ABI; handles exchanged over the group). ``local`` is this rank's
    buffer as a uint8 tensor; ``ptrs(offset)`` a device array of the P ranks' addresses."""

    def __init__(self, comm: "ShardComm", nbytes: int, device: torch.device):
        lib = _lib.load()
        hb = int(lib.ffb_p2p_handle_bytes())
        self.comm, self.nbytes, self.device = comm, nbytes, device
        self.base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * hb)()
        _lib.call("ffb_p2p_alloc", ctypes.c_size_t(nbytes), ctypes.byref(self.base), handle)
        mine = torch.tensor(list(handle), dtype=torch.uint8, device=device)
        everyone = torch.empty(comm.world * hb, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(everyone, mine, group=comm.group)
        everyone = everyone.view(comm.world, hb).cpu()
        self.addrs, self.opened = [], []
        for q in range(comm.world):
            if q == comm.rank:
                self.addrs.append(self.base.value)
                continue
            h = (ctypes.c_uint8 * hb)(*everyone[q].tolist())
            peer = ctypes.c_void_p()
            _lib.call("ffb_p2p_open", h, ctypes.byref(peer))
            self.addrs.append(peer.value)
            self.opened.append(peer)
        self.local = torch.as_tensor(_CudaArray(self.base.value, nbytes), device=device)

    def ptrs(self, offset: int = 0) -> Tensor:
        return torch.tensor([a + offset for a in self.addrs], dtype=torch.int64, device=self.device)

    def close(self) -> None:
        """Unmap the peers' buffers (every rank must do so before any rank frees its own)."""
        for peer in self.opened:
            _lib.call("ffb_p2p_close", peer)
        self.opened = []

    def free(self) -> None:
        """Free this rank's buffer (after every rank has closed its mapping of it)."""
        if self.base.value:
            self.local = None
            _lib.call("ffb_p2p_free", self.base)
            self.base = ctypes.c_void_p()


class _PeerExchange:
    """The NVLink peer-memory path of :class:`ShardComm` (one rank per GPU): transposes
    written by one kernel straight into the owning ranks' buffers (two buffers, alternated)
    and row gathers written into every rank's buffer, each followed by a bounded wait for
    the peers' writes (``ffb_shard_transpose_p2p`` / ``ffb_shard_gather_p2p`` /
    ``ffb_shard_wait_p2p``). Buffers are created on first use per shape, collectively (every
    rank runs the same schedule). A returned tensor aliases an exchange buffer: it is valid
    until the second-next exchange of its kind."""

    def __init__(self, comm: "ShardComm", device: torch.device):
        self.comm, self.device = comm, device
        p = comm.world
        self.flags = _PeerBuffer(comm, 256, device)   # P uint32 slots per rank
        self.flag_ptrs = self.flags.ptrs()
        self.sync = torch.zeros(2, dtype=torch.int32, device=device)  # arrival counter, epoch
        self.t_bufs: dict[tuple, tuple] = {}
        self.g_bufs: dict[tuple, tuple] = {}
        self.r_bufs: dict[tuple, tuple] = {}
        self.parity = 0
        assert p <= 8

    def _wait(self) -> None:
        _lib.call("ffb_shard_wait_p2p", _ptr(self.flags.local), _ptr(self.sync), self.comm.world,
                  self.comm.wait_limit_us, _stream())

    def transpose(self, x: Tensor) -> Tensor:
        r, n, c = x.shape
        key = (r, n, c, x.dtype)
        if key not in self.t_bufs:
            one = r * n * c * x.element_size()
            buf = _PeerBuffer(self.comm, 2 * one, self.device)
            self.t_bufs[key] = (buf, buf.ptrs(0), buf.ptrs(one), one)
        buf, p0, p1, one = self.t_bufs[key]
        b = self.parity
        self.parity ^= 1
        x = x.contiguous()
        _lib.call("ffb_shard_transpose_p2p", _ptr(x), _ptr(p1 if b else p0), _ptr(self.flag_ptrs), _ptr(self.sync),
                  r, n, self.comm.rank * r, self.comm.rank, self.comm.world, _stream())
        self.comm.mark("transpose_send")
        self._wait()
        return buf.local[b * one:(b + 1) * one].view(x.dtype).view(r, n, c)

    def gather_rows(self, x: Tensor) -> Tensor:
        x = x.contiguous()
        key = (tuple(x.shape), x.dtype)
        one = x.numel() * x.element_size()
        if key not in self.g_bufs:
            buf = _PeerBuffer(self.comm, self.comm.world * one, self.device)
            self.g_bufs[key] = (buf, buf.ptrs(0))
        buf, ptrs = self.g_bufs[key]
        _lib.call("ffb_shard_gather_p2p", _ptr(x), ctypes.c_size_t(one), _ptr(ptrs), _ptr(self.flag_ptrs),
                  _ptr(self.sync), self.comm.rank, self.comm.world, _stream())
        self.comm.mark("gather_send")
        self._wait()
        return buf.local.view(x.dtype).view((self.comm.world * x.shape[0],) + tuple(x.shape[1:]))

    def channel_rows(self, x: Tensor, mode: int, n: int, tag: str) -> Tensor:
        """The channel-sharded TriMul's scatters: mode 0 sends L or R rows ``[R][128][Np]`` to
        the channel owners (returns this rank's ``[C][N][Np]``, C = 128 / P); mode 1 sends U
        ``[C][N][Np]`` back to the row owners (returns this rank's ``[128][R][Np]``). ``tag``
        names the buffer (L, R and U each have their own)."""
        p = self.comm.world
        r, np_ = n // p, (n + 7) // 8 * 8
        shape = (128 // p, n, np_) if mode == 0 else (128, r, np_)
        key = (tag, shape)
        if key not in self.r_bufs:
            buf = _PeerBuffer(self.comm, shape[0] * shape[1] * shape[2] * 2, self.device)
            self.r_bufs[key] = (buf, buf.ptrs(0))
        buf, ptrs = self.r_bufs[key]
        x = x.contiguous()
        _lib.call("ffb_shard_rows_p2p", _ptr(x), mode, r, n, _ptr(ptrs), _ptr(self.flag_ptrs), _ptr(self.sync),
                  self.comm.rank, p, _stream())
        self.comm.mark(f"scatter_{tag}_send")
        self._wait()
        return buf.local.view(torch.bfloat16).view(shape)

    def buffers(self) -> list[_PeerBuffer]:
        return [b for b, *_ in list(self.t_bufs.values()) + list(self.g_bufs.values()) + list(self.r_bufs.values())] + [
            self.flags]


def device_identity(device: torch.device) -> tuple[str, str]:
    """``(host name, device UUID)`` of this rank's GPU: what decides whether two ranks can
    share memory over NVLink (same host) and whether their kernels may wait on one another
    (different devices)."""
    return socket.gethostname(), str(torch.cuda.get_device_properties(device).uuid)


def peer_path_allowed(identities: list[tuple[str, str]]) -> bool:
    """Whether ranks with these ``(host, device)`` identities may use the peer-memory
    exchanges: all on one host (CUDA IPC does not cross hosts), every rank on its own device
    (exchange kernels wait for the peers' kernels, which need not run concurrently on a
    shared GPU), at most 8 ranks."""
    hosts = {host for host, _ in identities}
    devices = [dev for _, dev in identities]
    return 1 < len(identities) <= 8 and len(hosts) == 1 and len(set(devices)) == len(devices)


class StageTimer:
    """CUDA events recorded on the current stream between the stages of sharded blocks; after
    a synchronize, :meth:`durations` sums the time between consecutive marks per stage name."""

    def __init__(self) -> None:
        self.marks: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append((name, ev))

    def durations(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for (_, a), (name, b) in zip(self.marks, self.marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


class ShardComm:
    """The two collectives of the schedule over one process group.

    With NCCL, one host and one GPU per rank (``peer="auto"``; checked once by gathering every
    rank's host name and device UUID) the exchanges run over NVLink peer memory
    (:class:`_PeerExchange`: one kernel writes each transpose / gather straight into the peers'
    buffers, then a wait bounded by ``wait_limit_us``, 0 = the library's 2 s); otherwise NCCL
    collectives on device tensors, or host copies for other backends (gloo). ``world == 1``
    (no group) makes both collectives local."""

    def __init__(self, group: dist.ProcessGroup | None = None, *, peer: str = "auto", trimul: str = "auto",
                 wait_limit_us: int = 0):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
            self.nccl = dist.get_backend(group) == "nccl"
        else:
            self.rank, self.world, self.nccl = 0, 1, False
        self.peer_mode = peer
        self.trimul_mode = trimul
        self.wait_limit_us = int(wait_limit_us)
        self._peer: _PeerExchange | None = None
        self._peer_ok: bool | None = None
        #: a :class:`StageTimer` to time the stages of the blocks run over this group (None: off)
        self.timer: StageTimer | None = None
        self.stage = ""

    def mark(self, name: str) -> None:
        """Record the end of stage ``name`` (prefixed by :attr:`stage`) when a timer is attached."""
        if self.timer is not None:
            self.timer.mark(f"{self.stage}{name}")

    def peer_capable(self, identity: tuple[str, str] | None = None) -> bool:
        """Collective (every rank calls it at the same point): gather each rank's
        :func:`device_identity` (or the given one) and decide :func:`peer_path_allowed`."""
        mine = identity if identity is not None else device_identity(torch.device("cuda", torch.cuda.current_device()))
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.group)
        return peer_path_allowed([tuple(x) for x in everyone])

    def _peer_path(self, x: Tensor) -> _PeerExchange | None:
        if self.peer_mode == "off" or self.world == 1 or not self.nccl or not x.is_cuda:
            return None
        if self._peer is None:
            if self._peer_ok is None:
                self._peer_ok = self.peer_capable()
            if not self._peer_ok:
                return None  # ranks on several hosts or sharing a GPU: NCCL collectives instead
            self._peer = _PeerExchange(self, x.device)
        return self._peer

    def trimul_by_channels(self, x: Tensor) -> bool:
        """Whether the TriMul contraction is sharded by channel: each rank receives L and R for
        its 128 / P channels over all rows and sends U back to the row owners, 3 (P - 1) / P of
        the pair per rank instead of the P - 1 rank chunks a gather of the right operand
        receives; the default for P >= 4 on the peer-memory path (``trimul="channels"`` /
        ``"rows"`` force either)."""
        if self.trimul_mode == "rows" or 128 % max(self.world, 1) or self._peer_path(x) is None:
            return False
        return self.trimul_mode == "channels" or self.world >= 4

    def close(self) -> None:
        """Release the peer-memory exchange buffers (collective: call on every rank, before the
        group is destroyed; tensors returned by the exchanges are invalid afterwards)."""
        if self._peer is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            bufs = self._peer.buffers()
            for buf in bufs:
                buf.close()
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # every rank has unmapped every peer buffer
            for buf in bufs:
                buf.free()
            self._peer = None

    def rows(self, n: int) -> tuple[int, int]:
        """(R, row0) of this rank for a pair of n rows (n must divide evenly)."""
        if n % self.world:
            raise ValueError(f"N={n} is not divisible by the {self.world} ranks of the group")
        r = n // self.world
        return r, self.rank * r

    def gather_rows(self, x: Tensor) -> Tensor:
        """Concatenate every rank's ``x`` along dim 0 (rank order)."""
        if self.world == 1:
            return x
        peer = self._peer_path(x)
        if peer is not None:
            return peer.gather_rows(x)
        if self.nccl or not x.is_cuda:
            out = torch.empty((self.world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
            return out
        host = x.detach().cpu().contiguous()
        out = torch.empty((self.world * host.shape[0],) + tuple(host.shape[1:]), dtype=host.dtype)
        dist.all_gather_into_tensor(out, host, group=self.group)
        return out.to(x.device)

    def transpose(self, x: Tensor) -> Tensor:
        """Rows [row0, row0 + R) of z -> the same rows of z^T (x: [R, N, c], N = world * R)."""
        if self.world == 1:
            return x.transpose(0, 1).contiguous()
        r, n, c = x.shape
        p = self.world
        peer = self._peer_path(x)
        if peer is not None and x.dtype == torch.bfloat16 and c == 128:
            return peer.transpose(x)
        # send[q] = x[:, q R : (q + 1) R] (the block of z^T rows that rank q holds)
        send = x.view(r, p, r, c).permute(1, 0, 2, 3).contiguous()
        if self.nccl or not x.is_cuda:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
        else:
            host = send.cpu()
            recv_h = torch.empty_like(host)
            dist.all_to_all_single(recv_h, host, group=self.group)
            recv = recv_h.to(x.device)
        # recv[q][i][a] = z[q R + i][row0 + a]  ->  y[a][q R + i]
        return recv.permute(2, 0, 1, 3).reshape(r, n, c).contiguous()


def swapped_trimul_weights(weights: dict[str, Tensor]) -> dict[str, Tensor]:
    """TriMul weights with the left / right projections and gates exchanged: incoming on z
    equals outgoing on z^T with these."""
    sw = dict(weights)
    for a, b in (("to_left.weight", "to_right.weight"), ("to_left_gate.weight", "to_right_gate.weight")):
        sw[a], sw[b] = weights[b], weights[a]
    return sw


# --------------------------------------------------------------------------- b200 shard ops
def _ptr(t: Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class B200ShardOps:
    """The row-sharded pieces on the sm_100a kernels (bf16 activations, master weights)."""

    def __init__(self, comm: ShardComm, masked_zero: bool = True):
        self.comm = comm
        self.masked = int(masked_zero)

    def trimul(self, z: Tensor, mask: Tensor, packed: Tensor) -> Tensor:
        r, n, _ = z.shape
        _, row0 = self.comm.rows(n)
        np_ = (n + 7) // 8 * 8
        dev = z.device
        left = torch.empty((r, 128, np_), dtype=torch.bfloat16, device=dev)
        right = torch.empty_like(left)
        zstats = torch.empty((r, n, 2), dtype=torch.float32, device=dev)
        _lib.call("ffb_trimul_shard_proj", _ptr(z), _ptr(mask), _ptr(packed), _ptr(left), _ptr(right), _ptr(zstats),
                  r, n, row0, _stream())
        self.comm.mark("proj")
        if self.comm.trimul_by_channels(z):
            peer = self.comm._peer
            cpp = 128 // self.comm.world
            lc = peer.channel_rows(left, 0, n, "L")
            rc = peer.channel_rows(right, 0, n, "R")
            self.comm.mark("exchange_LR")
            uc = torch.empty((cpp, n, np_), dtype=torch.bfloat16, device=dev)
            _lib.call("ffb_trimul_channel_contract", _ptr(lc), _ptr(rc), _ptr(uc), cpp, n, _stream())
            self.comm.mark("contract")
            u = peer.channel_rows(uc, 1, n, "U")
            self.comm.mark("exchange_U")
        else:
            right_all = self.comm.gather_rows(right)
            self.comm.mark("gather_R")
            u = torch.empty((128, r, np_), dtype=torch.bfloat16, device=dev)
            _lib.call("ffb_trimul_shard_contract", _ptr(left), _ptr(right_all), _ptr(u), r, n, _stream())
            self.comm.mark("contract")
        out = torch.empty_like(z)
        _lib.call("ffb_trimul_shard_out", _ptr(z), _ptr(mask), _ptr(packed), _ptr(u), _ptr(zstats), _ptr(None),
                  _ptr(out), r, n, row0, self.masked, _stream())
        self.comm.mark("out")
        return out

    def triattn(self, z: Tensor, mask: Tensor, packed: Tensor, *, transposed_bias: bool) -> Tensor:
        r, n, _ = z.shape
        _, row0 = self.comm.rows(n)
        np_ = (n + 7) // 8 * 8
        dev = z.device
        q = torch.empty((r, 4, n, 32), dtype=torch.bfloat16, device=dev)
        k = torch.empty_like(q)
        vt = torch.empty((r, 4, 32, np_), dtype=torch.bfloat16, device=dev)
        bias_rows = torch.empty((r, 4, np_), dtype=torch.bfloat16, device=dev)
        _lib.call("ffb_triattn_shard_proj", _ptr(z), _ptr(packed), _ptr(q), _ptr(k), _ptr(vt), _ptr(bias_rows), r, n,
                  _stream())
        self.comm.mark("proj")
        bias_all = self.comm.gather_rows(bias_rows)  # [N (rows of the pair held), 4, Np]
        if transposed_bias:
            # bias[q][h][k] = G[k][h][q]: the ending node's bias comes from the untransposed pair
            t = torch.zeros_like(bias_all)
            t[:, :, :n] = bias_all[:, :, :n].permute(2, 1, 0)
            bias_all = t
        self.comm.mark("gather_bias")
        o = torch.empty((r, n, 128), dtype=torch.bfloat16, device=dev)
        _lib.call("ffb_triattn_shard_attn", _ptr(q), _ptr(k), _ptr(vt), _ptr(bias_all), _ptr(mask), _ptr(o), r, n,
                  row0, _stream())
        self.comm.mark("attn")
        out = torch.empty_like(z)
        _lib.call("ffb_triattn_shard_out", _ptr(z), _ptr(mask), _ptr(packed), _ptr(o), _ptr(out), r, n, row0,
                  self.masked, _stream())
        self.comm.mark("out")
        return out

    def transition(self, z: Tensor, mask: Tensor, packed: Tensor) -> Tensor:
        r, n, _ = z.shape
        _, row0 = self.comm.rows(n)
        out = torch.empty_like(z)
        _lib.call("ffb_transition_shard_fwd", _ptr(z), _ptr(mask), _ptr(packed), _ptr(out), r, n, row0, self.masked,
                  _stream())
        self.comm.mark("transition")
        return out

    def single(self, s: Tensor, z: Tensor, mask: Tensor, apb_packed: Tensor, gate_bias: float,
               st_packed: Tensor) -> Tensor:
        """Attention with pair bias for this rank's query rows (their pair-bias rows are its own
        pair rows), an all-gather of the updated [R, 384] rows, then the single transition
        (replicated)."""
        from foldforge_b200 import kernels

        r, n, _ = z.shape
        row0 = self.comm.rows(n)[1]
        pb_rows = torch.empty((r, 16, n), dtype=torch.float32, device=z.device)
        _lib.call("ffb_apb_shard_pair_bias", _ptr(z), _ptr(apb_packed), _ptr(pb_rows), r, n, _stream())
        self.comm.mark("pair_bias")
        lib = _lib.load()
        ws = torch.empty(int(lib.ffb_apb_single_workspace_bytes(n)), dtype=torch.uint8, device=z.device)
        rows = torch.empty((r, s.shape[1]), dtype=s.dtype, device=s.device)
        _lib.call("ffb_apb_shard_single_rows", _ptr(s), _ptr(mask), _ptr(apb_packed), _ptr(pb_rows),
                  ctypes.c_float(gate_bias), _ptr(rows), _ptr(ws), ctypes.c_size_t(ws.numel()), n, row0, r,
                  self.masked, _stream())
        self.comm.mark("attention_rows")
        s2 = self.comm.gather_rows(rows)  # [N, 384]
        self.comm.mark("gather_rows")
        out = kernels.single_transition(s2[None], mask[None], st_packed, masked_zero=bool(self.masked))[0]
        self.comm.mark("transition")
        return out


# --------------------------------------------------------------------------- torch shard ops
def _ln(x: Tensor, w: Tensor | None, b: Tensor | None) -> Tensor:
    return F.layer_norm(x, x.shape[-1:], w, b, 1e-5)


def _lin(x: Tensor, w: Tensor) -> Tensor:
    return x @ w.t()


class TorchShardOps:
    """The same row-sharded pieces in fp32 torch (CPU or GPU): a check of the schedule."""

    def __init__(self, comm: ShardComm, masked_zero: bool = True):
        self.comm = comm
        self.masked_zero = masked_zero

    def _pair_mask(self, mask: Tensor, n: int) -> Tensor:
        r, row0 = self.comm.rows(n)
        m = mask.float()
        return m[row0:row0 + r, None] * m[None, :]  # [R, N]

    def trimul(self, z: Tensor, mask: Tensor, w: dict[str, Tensor]) -> Tensor:
        r, n, _ = z.shape
        pm = self._pair_mask(mask, n)[..., None]
        x = _ln(z, w["ln_pair.weight"], w["ln_pair.bias"])
        left = _lin(x, w["to_left.weight"]) * torch.sigmoid(_lin(x, w["to_left_gate.weight"])) * pm
        right = _lin(x, w["to_right.weight"]) * torch.sigmoid(_lin(x, w["to_right_gate.weight"])) * pm
        right_all = self.comm.gather_rows(right)  # [N, N, h]
        u = torch.einsum("ikc,jkc->ijc", left, right_all)
        delta = _lin(_ln(u, w["ln_out.weight"], w["ln_out.bias"]), w["to_out.weight"]) * torch.sigmoid(
            _lin(x, w["to_gate.weight"]))
        if self.masked_zero:
            delta = delta * pm
        return z + delta

    def triattn(self, z: Tensor, mask: Tensor, w: dict[str, Tensor], *, transposed_bias: bool) -> Tensor:
        r, n, c = z.shape
        h = w["to_bias.weight"].shape[0]
        d = w["to_query.weight"].shape[0] // h
        x = _ln(z, w["ln_pair.weight"], w["ln_pair.bias"])
        bias_all = self.comm.gather_rows(_lin(x, w["to_bias.weight"]))  # [N(q), N(k), H] of the pair held
        if transposed_bias:
            bias_all = bias_all.transpose(0, 1)
        bias = bias_all.permute(2, 0, 1)  # [H, q, k]

        def heads(t: Tensor) -> Tensor:  # [R, N, H*d] -> [R, H, N, d]
            return t.reshape(r, n, h, d).permute(0, 2, 1, 3)

        q = heads(_lin(x, w["to_query.weight"])) / d ** 0.5
        k = heads(_lin(x, w["to_key.weight"]))
        v = heads(_lin(x, w["to_value.weight"]))
        logits = q @ k.transpose(-1, -2) + bias[None]
        keep = self._pair_mask(mask, n)[:, None, None, :] > 0  # key mask of row i: m_i m_k
        logits = torch.where(keep, logits, torch.full_like(logits, -1e9))
        o = (logits.softmax(-1) @ v).permute(0, 2, 1, 3).reshape(r, n, h * d)
        delta = _lin(torch.sigmoid(_lin(x, w["to_gate.weight"])) * o, w["to_out.weight"])
        if self.masked_zero:
            delta = delta * self._pair_mask(mask, n)[..., None]
        return z + delta

    def transition(self, z: Tensor, mask: Tensor, w: dict[str, Tensor]) -> Tensor:
        x = _ln(z, w["ln_in.weight"], w["ln_in.bias"])
        delta = _lin(F.silu(_lin(x, w["expand_a.weight"])) * _lin(x, w["expand_b.weight"]), w["squeeze.weight"])
        if self.masked_zero:
            delta = delta * self._pair_mask(mask, z.shape[1])[..., None]
        return z + delta

    def single(self, s: Tensor, z: Tensor, mask: Tensor, wa: dict[str, Tensor], gate_bias: float,
               wt: dict[str, Tensor]) -> Tensor:
        r, n = z.shape[0], z.shape[1]
        row0 = self.comm.rows(n)[1]
        hs = wa["to_bias.weight"].shape[0]
        pb = _lin(_ln(z, wa["ln_pair.weight"], None), wa["to_bias.weight"])  # this rank's query rows [R, N, 16]
        y = _ln(s, wa["ln_single.weight"], wa["ln_single.bias"])
        cs = y.shape[-1]
        ds = cs // hs
        q = (_lin(y, wa["to_query.weight"]) + wa["to_query.bias"])[row0:row0 + r]
        k, v = _lin(y, wa["to_key.weight"]), _lin(y, wa["to_value.weight"])
        q = q.reshape(r, hs, ds).transpose(0, 1)
        k, v = (t.reshape(n, hs, ds).transpose(0, 1) for t in (k, v))
        logits = q @ k.transpose(-1, -2) / ds ** 0.5 + pb.permute(2, 0, 1)
        logits = torch.where(mask[None, None, :] > 0, logits, torch.full_like(logits, -1e9))
        o = (logits.softmax(-1) @ v).transpose(0, 1).reshape(r, cs)
        gate = _lin(y[row0:row0 + r], wa["to_gate.weight"])
        delta = _lin(torch.sigmoid(gate + gate_bias) * o, wa["to_out.weight"])
        if self.masked_zero:
            delta = delta * mask.float()[row0:row0 + r, None]
        s = self.comm.gather_rows(s[row0:row0 + r] + delta)
        x = _ln(s, wt["ln_in.weight"], wt["ln_in.bias"])
        d2 = _lin(F.silu(_lin(x, wt["expand_a.weight"])) * _lin(x, wt["expand_b.weight"]), wt["squeeze.weight"])
        if self.masked_zero:
            d2 = d2 * mask.float()[:, None]
        return s + d2


# --------------------------------------------------------------------------- the block
def _sub(state: dict[str, Tensor], prefix: str) -> dict[str, Tensor]:
    return {k[len(prefix) + 1:]: v for k, v in state.items() if k.startswith(prefix + ".")}


class ShardedPairformerBlock:
    """One AF3 Pairformer block over the row shards of a process group.

    ``block`` is an engine :class:`~foldforge_b200.engine.modules.PairformerBlock` (its
    weights are used, not its forward); ``ops`` is ``"b200"`` (the kernels; bf16 pair rows on
    the rank's GPU) or ``"torch"`` (fp32 restatement)."""

    def __init__(self, block, comm: ShardComm | None = None, *, ops: str = "b200", masked_zero: bool = True):
        self.comm = comm or ShardComm()
        self.ops_name = ops
        state = {k: v.detach() for k, v in block.state_dict().items()}
        self.gate_bias = float(getattr(block.single_attention, "gate_bias", 0.0))
        self.w = {name: _sub(state, name) for name in (
            "tri_multi_outgoing", "tri_multi_incoming", "tri_atten_starting", "tri_atten_ending",
            "transition_pair", "single_attention", "single_transition")}
        if "to_query.bias" not in self.w["single_attention"]:
            self.w["single_attention"]["to_query.bias"] = torch.zeros(
                self.w["single_attention"]["to_query.weight"].shape[0])
        # TriMul incoming runs as outgoing on z^T with left / right swapped
        self.w["tri_multi_incoming_t"] = swapped_trimul_weights(self.w["tri_multi_incoming"])
        if ops == "b200":
            self.ops = B200ShardOps(self.comm, masked_zero)
            self.packs: dict[str, Tensor] = {}
        elif ops == "torch":
            self.ops = TorchShardOps(self.comm, masked_zero)
        else:
            raise ValueError(f"unknown shard ops {ops!r}")

    def _pack(self, name: str, device: torch.device) -> Tensor:
        from foldforge_b200 import kernels

        if name not in self.packs:
            prep = {"tri_multi_outgoing": kernels.trimul_prepare, "tri_multi_incoming_t": kernels.trimul_prepare,
                    "tri_atten_starting": kernels.triattn_prepare, "tri_atten_ending": kernels.triattn_prepare,
                    "transition_pair": kernels.transition_prepare, "single_attention": kernels.apb_prepare,
                    "single_transition": kernels.single_transition_prepare}[name]
            self.packs[name] = prep(self.w[name], device)
        return self.packs[name]

    def _arg(self, name: str, device: torch.device):
        return self._pack(name, device) if self.ops_name == "b200" else self.w[name]

    def __call__(self, z: Tensor, mask: Tensor, s: Tensor) -> tuple[Tensor, Tensor]:
        """z: this rank's pair rows ``[R, N, 128]``; mask ``[N]`` (bool / uint8, all tokens);
        s ``[N, 384]`` (replicated). Returns the updated rows and single."""
        comm, ops, dev = self.comm, self.ops, z.device
        if self.ops_name == "b200":
            mask = mask.to(torch.uint8).contiguous()
        a = lambda name: self._arg(name, dev)  # noqa: E731

        def stage(name: str) -> None:
            comm.stage = name

        stage("TMo.")
        z = ops.trimul(z, mask, a("tri_multi_outgoing"))
        y = comm.transpose(z)
        stage("")
        comm.mark("transpose")
        stage("TMi.")
        y = ops.trimul(y, mask, a("tri_multi_incoming_t"))
        z = comm.transpose(y)
        stage("")
        comm.mark("transpose")
        stage("TAs.")
        z = ops.triattn(z, mask, a("tri_atten_starting"), transposed_bias=False)
        y = comm.transpose(z)
        stage("")
        comm.mark("transpose")
        stage("TAe.")
        y = ops.triattn(y, mask, a("tri_atten_ending"), transposed_bias=True)
        stage("pair.")
        y = ops.transition(y, mask, a("transition_pair"))
        z = comm.transpose(y)
        stage("")
        comm.mark("transpose")
        stage("single.")
        s = ops.single(s, z, mask, a("single_attention"), self.gate_bias, a("single_transition"))
        stage("")
        return z, s
