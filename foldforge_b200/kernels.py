"""Torch-facing wrappers of the C ABI: tensors in, tensors out, on the current stream.

These wrappers only check tensors and pass raw pointers; all arithmetic runs in the
sm_100a kernels of ``_ffb.so``. A tensor on the CPU, of another dtype or with an
unsupported layout is refused with :class:`~foldforge_b200._lib.UnsupportedCall`
before anything is launched.
"""

from __future__ import annotations

import ctypes

import torch

from foldforge_b200 import _lib

Tensor = torch.Tensor
BF16, F32 = 0, 1
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2
_DTYPES = {torch.bfloat16: BF16, torch.float32: F32}


def _ptr(t: Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need_cuda(*ts: Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.UnsupportedCall("foldforge_b200", 2, "tensor is not on a CUDA device")


def layer_norm(x: Tensor, weight: Tensor | None, bias: Tensor | None, eps: float = 1e-5) -> Tensor:
    """LayerNorm over the last axis (fp32 affine), output in ``x.dtype``."""
    _need_cuda(x, weight, bias)
    if x.dtype not in _DTYPES:
        raise _lib.UnsupportedCall("layer_norm", 2, f"dtype {x.dtype}")
    x = x.contiguous()
    y = torch.empty_like(x)
    c = x.shape[-1]
    w = None if weight is None else weight.detach().float().contiguous()
    b = None if bias is None else bias.detach().float().contiguous()
    _lib.call("ffb_layernorm_fwd", _ptr(x), _ptr(y), _ptr(w), _ptr(b), x.numel() // c, c, ctypes.c_float(eps),
              _DTYPES[x.dtype], _stream())
    return y


def gemm_nt(
    a: Tensor,
    b: Tensor,
    *,
    bias: Tensor | None = None,
    epilogue: int = EPI_STORE,
    residual: Tensor | None = None,
    row_mask: Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out: Tensor | None = None,
) -> Tensor:
    """``a @ b.T`` on the tensor cores: ``a [.., m, k]``, ``b [.., n, k]`` bf16 (same batch
    shape or ``b`` 2-D), fp32 accumulation, output ``out_dtype``."""
    _need_cuda(a, b, bias, residual, row_mask)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise _lib.UnsupportedCall("gemm_nt", 2, "operands must be bf16")
    a = a.contiguous()
    b = b.contiguous()
    k = a.shape[-1]
    n = b.shape[-2]
    if b.dim() == 2:  # shared weight: fold every leading axis of a into the rows
        m, batch, sb = a.numel() // k, 1, 0
    else:
        m = a.shape[-2]
        batch = a.numel() // (m * k)
        sb = n * k
    n_out = n // 2 if epilogue == EPI_SWIGLU else n
    if out is None:
        out = torch.empty(*a.shape[:-1], n_out, device=a.device, dtype=out_dtype)
    if residual is not None:
        residual = residual.contiguous()
    mask = None if row_mask is None else row_mask.to(torch.uint8).contiguous()
    _lib.call(
        "ffb_gemm_bf16_nt", _ptr(a), _ptr(b), _ptr(out), batch, m, n, k, k, k, n_out, m * k, sb, m * n_out,
        _DTYPES[out.dtype], _ptr(None if bias is None else bias.float().contiguous()), epilogue, _ptr(residual),
        _ptr(mask), _stream(),
    )
    return out


def _f32(t: Tensor) -> Tensor:
    return t.detach().to(torch.float32).contiguous()


def trimul_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack a ``TriangleMultiplication``'s fp32 weights (engine keys) for the kernels."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_trimul_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_pair.weight", "ln_pair.bias", "ln_out.weight", "ln_out.bias", "to_left.weight", "to_right.weight",
            "to_left_gate.weight", "to_right_gate.weight", "to_out.weight", "to_gate.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_trimul_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts  # the pack kernel reads them asynchronously
    return packed


def _mask_u8(mask: Tensor) -> Tensor:
    if mask.dtype == torch.bool and mask.is_contiguous():
        return mask.view(torch.uint8)  # same bytes, no cast kernel
    return mask.to(torch.uint8).contiguous()


def trimul(z: Tensor, mask: Tensor, packed: Tensor, *, outgoing: bool, masked_zero: bool = True,
           stages: int = 7, workspace: Tensor | None = None, out: Tensor | None = None) -> Tensor:
    """Triangle multiplicative update with residual: ``z [B, N, N, 128]`` bf16, ``mask [B, N]``.
    ``stages`` / ``workspace`` / ``out`` select and reuse buffers for a subset of its launches."""
    _need_cuda(z, mask, packed)
    if z.dtype != torch.bfloat16 or z.dim() != 4 or z.shape[-1] != 128:
        raise _lib.UnsupportedCall("trimul", 2, f"needs bf16 [B, N, N, 128], got {z.dtype} {tuple(z.shape)}")
    z = z.contiguous()
    b, n = z.shape[0], z.shape[1]
    lib = _lib.load()
    ws_bytes = int(lib.ffb_trimul_workspace_bytes(b, n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=z.device) if workspace is None else workspace
    out = torch.empty_like(z) if out is None else out
    m = _mask_u8(mask)
    _lib.call("ffb_trimul_fwd_stages", _ptr(z), _ptr(m), _ptr(packed), _ptr(out), _ptr(ws), ctypes.c_size_t(ws.numel()),
              b, n, int(outgoing), int(masked_zero), stages, _stream())
    return out


def triattn_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack a ``TriangleAttention`` (AF3)'s fp32 weights (engine keys) for the kernels."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_triattn_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_pair.weight", "ln_pair.bias", "to_bias.weight", "to_query.weight", "to_key.weight",
            "to_value.weight", "to_gate.weight", "to_out.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_triattn_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def triattn(z: Tensor, mask: Tensor, packed: Tensor, *, starting: bool, masked_zero: bool = True,
            stages: int = 7, workspace: Tensor | None = None, out: Tensor | None = None) -> Tensor:
    """Triangle attention with residual: ``z [B, N, N, 128]`` bf16, ``mask [B, N]``."""
    _need_cuda(z, mask, packed)
    if z.dtype != torch.bfloat16 or z.dim() != 4 or z.shape[-1] != 128:
        raise _lib.UnsupportedCall("triattn", 2, f"needs bf16 [B, N, N, 128], got {z.dtype} {tuple(z.shape)}")
    z = z.contiguous()
    b, n = z.shape[0], z.shape[1]
    lib = _lib.load()
    ws_bytes = int(lib.ffb_triattn_workspace_bytes(b, n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=z.device) if workspace is None else workspace
    out = torch.empty_like(z) if out is None else out
    m = _mask_u8(mask)
    _lib.call("ffb_triattn_fwd_stages", _ptr(z), _ptr(m), _ptr(packed), _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, n, int(starting), int(masked_zero), stages, _stream())
    return out


def transition_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack a pair ``Transition(128, 4)``'s fp32 weights (engine keys) for the fused kernel."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_transition_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_in.weight", "ln_in.bias", "expand_a.weight", "expand_b.weight", "squeeze.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_transition_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def transition(z: Tensor, mask: Tensor | None, packed: Tensor, *, masked_zero: bool = True) -> Tensor:
    """Fused pair transition with residual: ``z [B, N, N, 128]`` bf16."""
    _need_cuda(z, mask, packed)
    if z.dtype != torch.bfloat16 or z.dim() != 4 or z.shape[-1] != 128:
        raise _lib.UnsupportedCall("transition", 2, f"needs bf16 [B, N, N, 128], got {z.dtype} {tuple(z.shape)}")
    z = z.contiguous()
    out = torch.empty_like(z)
    m = None if mask is None else _mask_u8(mask)
    _lib.call("ffb_transition_fwd", _ptr(z), _ptr(m), _ptr(packed), _ptr(out), z.shape[0], z.shape[1],
              int(masked_zero and m is not None), _stream())
    return out


def apb_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack an ``AttentionPairBias``'s fp32 weights (engine keys) for the kernels."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_apb_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_single.weight", "ln_single.bias", "to_query.weight", "to_query.bias", "to_key.weight",
            "to_value.weight", "to_gate.weight", "to_out.weight", "ln_pair.weight", "to_bias.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_apb_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def attention_pair_bias(s: Tensor, z: Tensor, mask: Tensor, packed: Tensor, *, extra_pair_bias: Tensor | None = None,
                        gate_bias: float = 0.0, masked_zero: bool = True) -> Tensor:
    """Single attention with pair bias and residual: ``s [B, N, 384]``, ``z [B, N, N, 128]`` bf16."""
    _need_cuda(s, z, mask, packed, extra_pair_bias)
    if s.dtype != torch.bfloat16 or z.dtype != torch.bfloat16 or s.shape[-1] != 384 or z.shape[-1] != 128:
        raise _lib.UnsupportedCall("attention_pair_bias", 2, "needs bf16 s [B, N, 384] and z [B, N, N, 128]")
    s, z = s.contiguous(), z.contiguous()
    b, n = s.shape[0], s.shape[1]
    lib = _lib.load()
    ws_bytes = int(lib.ffb_apb_workspace_bytes(b, n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=s.device)
    out = torch.empty_like(s)
    extra = None
    extra_dtype = BF16
    if extra_pair_bias is not None:
        extra = extra_pair_bias.expand(b, 16, n, n).contiguous()
        if extra.dtype not in (torch.bfloat16, torch.float32):
            extra = extra.float()
        extra_dtype = _DTYPES[extra.dtype]
    _lib.call("ffb_apb_fwd", _ptr(s), _ptr(z), _ptr(_mask_u8(mask)), _ptr(packed), _ptr(extra), extra_dtype,
              ctypes.c_float(gate_bias), _ptr(out), _ptr(ws), ctypes.c_size_t(ws_bytes), b, n, int(masked_zero),
              _stream())
    return out


def single_transition_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack a single ``Transition(384, 4)``'s fp32 weights for the GEMM path."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_single_transition_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_in.weight", "ln_in.bias", "expand_a.weight", "expand_b.weight", "squeeze.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_single_transition_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def single_transition(s: Tensor, mask: Tensor | None, packed: Tensor, *, masked_zero: bool = True) -> Tensor:
    """Single transition with residual: ``s [B, N, 384]`` bf16."""
    _need_cuda(s, mask, packed)
    if s.dtype != torch.bfloat16 or s.shape[-1] != 384:
        raise _lib.UnsupportedCall("single_transition", 2, "needs bf16 [B, N, 384]")
    s = s.contiguous()
    b, n = s.shape[0], s.shape[1]
    lib = _lib.load()
    ws_bytes = int(lib.ffb_single_transition_workspace_bytes(b, n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=s.device)
    out = torch.empty_like(s)
    m = None if mask is None else _mask_u8(mask)
    _lib.call("ffb_single_transition_fwd", _ptr(s), _ptr(m), _ptr(packed), _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws_bytes), b, n, int(masked_zero and m is not None), _stream())
    return out


# --------------------------------------------------------------------------- fp32 / any-width path
# The FP32 SIMT kernels of csrc/generic.cu: fp32 activations (the "fp32" precision), and any
# widths (e.g. c_z = 64). Weights are the module's fp32 matrices as they are ([out, in]).
def _weight_ptrs(weights: dict[str, Tensor], keys: tuple[str, ...], device: torch.device):
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    table = (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])  # a host array of device pointers
    return ctypes.cast(table, ctypes.c_void_p), (ts, table)


def _f32_input(x: Tensor, name: str) -> Tensor:
    if x.dtype != torch.float32:
        raise _lib.UnsupportedCall(name, 2, f"the fp32 path takes fp32 activations, got {x.dtype}")
    return x.contiguous()


def _workspace(nbytes: int, device: torch.device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def trimul_f32(z: Tensor, mask: Tensor, weights: dict[str, Tensor], *, outgoing: bool,
               masked_zero: bool = True) -> Tensor:
    """Triangle multiplicative update with residual in fp32: ``z [B, N, N, c]``, any c / hidden."""
    _need_cuda(z, mask)
    z = _f32_input(z, "trimul_f32")
    b, n, c = z.shape[0], z.shape[1], z.shape[-1]
    h = weights["to_left.weight"].shape[0]
    keys = ("ln_pair.weight", "ln_pair.bias", "ln_out.weight", "ln_out.bias", "to_left.weight", "to_right.weight",
            "to_left_gate.weight", "to_right_gate.weight", "to_out.weight", "to_gate.weight")
    ptrs, keep = _weight_ptrs(weights, keys, z.device)
    lib = _lib.load()
    ws = _workspace(lib.ffb_trimul_f32_workspace_bytes(b, n, c, h), z.device)
    out = torch.empty_like(z)
    _lib.call("ffb_trimul_fwd_f32", _ptr(z), _ptr(_mask_u8(mask)), ptrs, _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, n, c, h, int(outgoing), int(masked_zero), _stream())
    del keep
    return out


def triattn_f32(z: Tensor, mask: Tensor, weights: dict[str, Tensor], *, starting: bool, n_head: int,
                masked_zero: bool = True) -> Tensor:
    """Triangle attention with residual in fp32: ``z [B, N, N, c]``, any heads x width <= 64."""
    _need_cuda(z, mask)
    z = _f32_input(z, "triattn_f32")
    b, n, c = z.shape[0], z.shape[1], z.shape[-1]
    d = weights["to_query.weight"].shape[0] // n_head
    keys = ("ln_pair.weight", "ln_pair.bias", "to_bias.weight", "to_query.weight", "to_key.weight",
            "to_value.weight", "to_gate.weight", "to_out.weight")
    ptrs, keep = _weight_ptrs(weights, keys, z.device)
    lib = _lib.load()
    ws = _workspace(lib.ffb_triattn_f32_workspace_bytes(b, n, c, n_head, d), z.device)
    out = torch.empty_like(z)
    _lib.call("ffb_triattn_fwd_f32", _ptr(z), _ptr(_mask_u8(mask)), ptrs, _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, n, c, n_head, d, int(starting), int(masked_zero), _stream())
    del keep
    return out


def transition_f32(x: Tensor, mask: Tensor | None, weights: dict[str, Tensor], *, masked_zero: bool = True) -> Tensor:
    """Transition with residual in fp32: pair ``[B, N, N, c]`` or single ``[B, N, c]``, any c and factor."""
    _need_cuda(x, mask)
    x = _f32_input(x, "transition_f32")
    pair = x.dim() == 4
    b, n, c = x.shape[0], x.shape[1], x.shape[-1]
    factor = weights["expand_a.weight"].shape[0] // c
    if mask is None:
        mask, masked_zero = torch.ones(b, n, dtype=torch.bool, device=x.device), False
    keys = ("ln_in.weight", "ln_in.bias", "expand_a.weight", "expand_b.weight", "squeeze.weight")
    ptrs, keep = _weight_ptrs(weights, keys, x.device)
    lib = _lib.load()
    rows = b * n * (n if pair else 1)
    ws = _workspace(lib.ffb_transition_f32_workspace_bytes(rows, c, factor), x.device)
    out = torch.empty_like(x)
    _lib.call("ffb_transition_fwd_f32", _ptr(x), _ptr(_mask_u8(mask)), ptrs, _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, n, c, factor, int(pair), int(masked_zero), _stream())
    del keep
    return out


def attention_pair_bias_f32(s: Tensor, z: Tensor, mask: Tensor, weights: dict[str, Tensor], *, n_head: int,
                            extra_pair_bias: Tensor | None = None, gate_bias: float = 0.0,
                            masked_zero: bool = True) -> Tensor:
    """Single attention with pair bias and residual in fp32: ``s [B, N, c_s]``, ``z [B, N, N, c_z]``."""
    _need_cuda(s, z, mask, extra_pair_bias)
    s, z = _f32_input(s, "apb_f32"), _f32_input(z, "apb_f32")
    b, n, cs, cz = s.shape[0], s.shape[1], s.shape[-1], z.shape[-1]
    w = dict(weights)
    if w.get("to_query.bias") is None:
        w["to_query.bias"] = torch.zeros(cs, device=s.device)
    keys = ("ln_single.weight", "ln_single.bias", "to_query.weight", "to_query.bias", "to_key.weight",
            "to_value.weight", "to_gate.weight", "to_out.weight", "ln_pair.weight", "to_bias.weight")
    ptrs, keep = _weight_ptrs(w, keys, s.device)
    extra = None
    if extra_pair_bias is not None:
        extra = extra_pair_bias.float().expand(b, n_head, n, n).contiguous()
    lib = _lib.load()
    ws = _workspace(lib.ffb_apb_f32_workspace_bytes(b, n, cs, cz, n_head), s.device)
    out = torch.empty_like(s)
    _lib.call("ffb_apb_fwd_f32", _ptr(s), _ptr(z), _ptr(_mask_u8(mask)), ptrs, _ptr(extra), ctypes.c_float(gate_bias),
              _ptr(out), _ptr(ws), ctypes.c_size_t(ws.numel()), b, n, cs, cz, n_head, int(masked_zero), _stream())
    del keep
    return out


# --------------------------------------------------------------------------- MSA module (csrc/msa.cu)
def opm_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack an ``OuterProductMean`` (AF3 form: c_m 64, 32 channels a side, c_z 128)'s fp32 weights."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_opm_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_msa.weight", "ln_msa.bias", "to_left.weight", "to_right.weight", "to_out.weight", "to_out.bias")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_opm_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def outer_product_mean(msa: Tensor, row_mask: Tensor, packed: Tensor, *, count_offset: float | None) -> Tensor:
    """The outer product mean's raw update ``[B, N, N, 128]`` bf16 from ``msa [B, S, N, 64]`` bf16 and
    the MSA row mask ``[B, S, N]``; divisor ``n + count_offset`` (``None``: ``max(n, 1)``)."""
    _need_cuda(msa, row_mask, packed)
    if msa.dtype != torch.bfloat16 or msa.dim() != 4 or msa.shape[-1] != 64:
        raise _lib.UnsupportedCall("outer_product_mean", 2, f"needs bf16 [B, S, N, 64], got {msa.dtype} {tuple(msa.shape)}")
    msa = msa.contiguous()
    b, s, n = msa.shape[:3]
    lib = _lib.load()
    ws = _workspace(lib.ffb_opm_workspace_bytes(s, n), msa.device)
    delta = torch.empty((b, n, n, 128), dtype=torch.bfloat16, device=msa.device)
    offset = -1.0 if count_offset is None else float(count_offset)
    _lib.call("ffb_opm_fwd", _ptr(msa), _ptr(_mask_u8(row_mask)), _ptr(packed), _ptr(delta), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, s, n, ctypes.c_float(offset), _stream())
    return delta


def pwa_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """Pack an ``MSAPairWeightedAveraging`` (c_m 64, c_z 128, 8 heads x 8)'s fp32 weights."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_pwa_packed_bytes()), dtype=torch.uint8, device=device)
    keys = ("ln_msa.weight", "ln_msa.bias", "ln_pair.weight", "to_bias.weight", "to_value.weight", "to_gate.weight",
            "to_out.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_pwa_prepare", *[_ptr(t) for t in ts], _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def pair_weighted_averaging(msa: Tensor, pair: Tensor, key_mask: Tensor, packed: Tensor) -> Tensor:
    """``msa + PWA(msa, pair)``: ``msa [B, S, N, 64]``, ``pair [B, N, N, 128]`` bf16, ``key_mask [B, N]``
    (a column is a key when some MSA row has it)."""
    _need_cuda(msa, pair, key_mask, packed)
    if msa.dtype != torch.bfloat16 or pair.dtype != torch.bfloat16 or msa.shape[-1] != 64 or pair.shape[-1] != 128:
        raise _lib.UnsupportedCall("pair_weighted_averaging", 2, "needs bf16 msa [B, S, N, 64] and pair [B, N, N, 128]")
    msa, pair = msa.contiguous(), pair.contiguous()
    b, s, n = msa.shape[:3]
    lib = _lib.load()
    ws = _workspace(lib.ffb_pwa_workspace_bytes(s, n), msa.device)
    out = torch.empty_like(msa)
    _lib.call("ffb_pwa_fwd", _ptr(msa), _ptr(pair), _ptr(_mask_u8(key_mask)), _ptr(packed), _ptr(out), _ptr(ws),
              ctypes.c_size_t(ws.numel()), b, s, n, _stream())
    return out


def transition_gemm_prepare(weights: dict[str, Tensor], c: int, n: int, device: torch.device) -> Tensor:
    """Pack a ``Transition(c, n)`` for the tensor-core transition of any width (c a multiple of 8)."""
    lib = _lib.load()
    packed = torch.empty(int(lib.ffb_transition_gemm_packed_bytes(c, n)), dtype=torch.uint8, device=device)
    keys = ("ln_in.weight", "ln_in.bias", "expand_a.weight", "expand_b.weight", "squeeze.weight")
    ts = [_f32(weights[k]).to(device) for k in keys]
    _need_cuda(*ts)
    _lib.call("ffb_transition_gemm_prepare", *[_ptr(t) for t in ts], c, n, _ptr(packed), _stream())
    packed._keepalive = ts
    return packed


def transition_gemm(x: Tensor, packed: Tensor, c: int, n: int) -> Tensor:
    """Unmasked transition with residual over the rows of ``x [..., c]`` bf16 on the tensor cores."""
    _need_cuda(x, packed)
    if x.dtype != torch.bfloat16 or x.shape[-1] != c:
        raise _lib.UnsupportedCall("transition_gemm", 2, f"needs bf16 [..., {c}], got {x.dtype} {tuple(x.shape)}")
    x = x.contiguous()
    rows = x.numel() // c
    lib = _lib.load()
    ws = _workspace(lib.ffb_transition_gemm_workspace_bytes(rows, c, n), x.device)
    out = torch.empty_like(x)
    _lib.call("ffb_transition_gemm_fwd", _ptr(x), _ptr(packed), _ptr(out), _ptr(ws), ctypes.c_size_t(ws.numel()),
              ctypes.c_int64(rows), c, n, _stream())
    return out


# --------------------------------------------------------------------------- diffusion transformer
#: the 23 weights of a token DiT block in the order ``ffb_dit_prepare`` takes them
DIT_WEIGHTS = (
    "attention.ada_ln_in.ln_cond.weight", "attention.ada_ln_in.to_scale.weight", "attention.ada_ln_in.to_scale.bias",
    "attention.ada_ln_in.to_bias.weight", "attention.to_query.weight", "attention.to_query.bias",
    "attention.to_key.weight", "attention.to_value.weight", "attention.to_gate.weight", "attention.to_scale.weight",
    "attention.to_scale.bias", "attention.to_out.weight", "attention.ln_pair.weight", "attention.to_bias.weight",
    "transition.ada_ln_in.ln_cond.weight", "transition.ada_ln_in.to_scale.weight",
    "transition.ada_ln_in.to_scale.bias", "transition.ada_ln_in.to_bias.weight", "transition.expand_a.weight",
    "transition.expand_b.weight", "transition.squeeze.weight", "transition.to_scale.weight",
    "transition.to_scale.bias",
)


def dit_prepare(weights: dict[str, Tensor], device: torch.device) -> Tensor:
    """The packed image of one token DiT block (AF3 widths) from its fp32 engine-key weights."""
    lib = _lib.load()
    ptrs, keep = _weight_ptrs(weights, DIT_WEIGHTS, device)
    packed = torch.empty(int(lib.ffb_dit_packed_bytes()), dtype=torch.uint8, device=device)
    _lib.call("ffb_dit_prepare", ptrs, _ptr(packed), _stream())
    del keep
    return packed


def dit_condition(cond: Tensor, pair: Tensor, packed: Tensor) -> Tensor:
    """The block's per-fold tables (AdaLN scale / shift, output gates, pair logits) from
    ``cond [L, 384]`` and ``pair [L, L, 128]`` (bf16)."""
    _need_cuda(cond, pair, packed)
    if cond.dtype != torch.bfloat16 or pair.dtype != torch.bfloat16:
        raise _lib.UnsupportedCall("ffb_dit_condition", 2, f"bf16 conditioning, got {cond.dtype} / {pair.dtype}")
    cond, pair = cond.contiguous(), pair.contiguous()
    n = cond.shape[0]
    lib = _lib.load()
    tables = torch.empty(int(lib.ffb_dit_tables_bytes(n)), dtype=torch.uint8, device=cond.device)
    ws = _workspace(lib.ffb_dit_condition_workspace_bytes(n), cond.device)
    _lib.call("ffb_dit_condition", _ptr(cond), _ptr(pair), _ptr(packed), _ptr(tables), _ptr(ws),
              ctypes.c_size_t(ws.numel()), n, _stream())
    return tables


def dit_forward(x: Tensor, mask: Tensor, packed: Tensor, tables: Tensor, *, workspace: Tensor | None = None,
                out: Tensor | None = None) -> Tensor:
    """One token DiT block on ``x [S, L, 768]`` (bf16) with the fold's tables; ``mask [L]``."""
    _need_cuda(x, mask, packed, tables)
    if x.dtype != torch.bfloat16:
        raise _lib.UnsupportedCall("ffb_dit_fwd", 2, f"bf16 activations, got {x.dtype}")
    x = x.contiguous()
    s, n = x.shape[0], x.shape[1]
    lib = _lib.load()
    if workspace is None:
        workspace = _workspace(lib.ffb_dit_workspace_bytes(s, n), x.device)
    if out is None:
        out = torch.empty_like(x)
    _lib.call("ffb_dit_fwd", _ptr(x), _ptr(_mask_u8(mask)), _ptr(packed), _ptr(tables), _ptr(out), _ptr(workspace),
              ctypes.c_size_t(workspace.numel()), s, n, _stream())
    return out
