"""CPU restatement of the reference's Pairformer block equations (test oracle).

Every function takes unbatched tensors (``z [N, N, c]``, ``s [N, c_s]``), a token mask
``tokens [N]`` (1 = real token, 0 = padding) and a parameter mapping ``p`` keyed by the
engine state-dict names of ONE op (e.g. ``"to_left.weight"``), and returns the op's
output WITH its residual, as the engine classes do. The pair mask of the reference graph
is the outer product ``tokens[:, None] * tokens[None, :]`` (``modules/engine/modules.py:
241-265``); every masked position is computed by the same equations as a real one, which
is what the reference does (its parity test only compares real positions).

Arithmetic is done in ``dtype`` (float32 by default; float64 for a tighter truth).
Reference citations are paths inside the FoldForge source tree.
"""

from __future__ import annotations

from collections.abc import Mapping

import torch

Tensor = torch.Tensor
Params = Mapping[str, Tensor]

#: ``attention(mask_value=-1e9)``: masked logits are REPLACED by this value
#: (``legacy/reference/attention.py:14-54``, ``masked_fill``), so a fully masked row
#: softmaxes to uniform weights.
MASK_VALUE = -1e9
LN_EPS = 1e-5


def _p(p: Params, key: str, dtype: torch.dtype) -> Tensor:
    return p[key].to(dtype)


def layer_norm(x: Tensor, weight: Tensor | None, bias: Tensor | None, eps: float = LN_EPS) -> Tensor:
    """``torch.nn.LayerNorm`` over the last axis (biased variance, eps inside the root)."""
    mean = x.mean(-1, keepdim=True)
    var = (x - mean).square().mean(-1, keepdim=True)
    y = (x - mean) / torch.sqrt(var + eps)
    if weight is not None:
        y = y * weight
    if bias is not None:
        y = y + bias
    return y


def _linear(x: Tensor, w: Tensor, b: Tensor | None = None) -> Tensor:
    y = x @ w.T
    return y if b is None else y + b


def _pair_mask(tokens: Tensor, dtype: torch.dtype) -> Tensor:
    t = tokens.to(dtype)
    return t[:, None] * t[None, :]


def triangle_multiplication(
    z: Tensor, tokens: Tensor, p: Params, *, outgoing: bool, dtype: torch.dtype = torch.float32
) -> Tensor:
    """Triangle multiplicative update, residual included.

    Follows ``legacy/reference/triangle.py:19-50`` (``triangle_update``) bound by
    ``legacy/routing.py:44-54,82-102`` (``triangle_residual``): the projection is masked
    by the pair mask, then multiplied by the sigmoid gate; outgoing contracts
    ``u_ij = sum_k L_ik R_jk``, incoming ``u_ij = sum_k L_ki R_kj`` (the engine's left /
    right after the converter's interleave, ``legacy/released.py:135-173``); the centre
    LayerNorm, output projection and output gate follow.
    """
    z = z.to(dtype)
    x = layer_norm(z, _p(p, "ln_pair.weight", dtype), _p(p, "ln_pair.bias", dtype))
    m = _pair_mask(tokens, dtype)[..., None]
    left = _linear(x, _p(p, "to_left.weight", dtype)) * m
    left = left * torch.sigmoid(_linear(x, _p(p, "to_left_gate.weight", dtype)))
    right = _linear(x, _p(p, "to_right.weight", dtype)) * m
    right = right * torch.sigmoid(_linear(x, _p(p, "to_right_gate.weight", dtype)))
    if outgoing:
        u = torch.einsum("ikc,jkc->ijc", left, right)
    else:
        u = torch.einsum("kic,kjc->ijc", left, right)
    u = layer_norm(u, _p(p, "ln_out.weight", dtype), _p(p, "ln_out.bias", dtype))
    delta = _linear(u, _p(p, "to_out.weight", dtype))
    delta = delta * torch.sigmoid(_linear(x, _p(p, "to_gate.weight", dtype)))
    return z + delta


def _masked_softmax_attention(q: Tensor, k: Tensor, v: Tensor, bias: Tensor | None, keep: Tensor) -> Tensor:
    """``softmax(q k^T * d^-1/2 + bias, masked_fill(~keep, -1e9)) v`` over the last two axes.

    ``legacy/reference/attention.py:14-54`` (``attention``) as called by
    ``dot_product_attention`` (``:77-100``, scale ``d ** -0.5``): the bias is added
    BEFORE the mask replaces logits.
    """
    logits = (q * q.shape[-1] ** -0.5) @ k.transpose(-1, -2)
    if bias is not None:
        logits = logits + bias
    logits = logits.masked_fill(~keep, MASK_VALUE)
    return logits.softmax(-1) @ v


def triangle_attention(
    z: Tensor,
    tokens: Tensor,
    p: Params,
    *,
    starting: bool,
    n_head: int = 4,
    dtype: torch.dtype = torch.float32,
) -> Tensor:
    """Triangle attention around the starting (rows) or ending (columns) node.

    ``legacy/attention.py:108-171`` (``GridSelfAttention``) with AF3 settings
    (``spec.py:125`` untransposed pair bias, ``:437`` no projection biases, ``:470``
    output turned back): the bias ``b_h,qk = W_b LN(z)_qk`` is computed on the
    UNtransposed pair and indexed by (query, key) in both directions; the ending node runs
    the same attention on ``z^T`` and transposes the result back. The key mask of row
    ``r`` is the pair mask ``m_r m_k`` (``legacy/reference/attention.py:88-92``).
    """
    z = z.to(dtype)
    n = z.shape[0]
    x = layer_norm(z, _p(p, "ln_pair.weight", dtype), _p(p, "ln_pair.bias", dtype))
    bias = _linear(x, _p(p, "to_bias.weight", dtype)).permute(2, 0, 1)  # [H, q, k]
    if not starting:
        x = x.transpose(0, 1)
    hidden = _p(p, "to_query.weight", dtype).shape[0]
    d = hidden // n_head

    def heads(t: Tensor) -> Tensor:  # [rows, n, H*d] -> [rows, H, n, d]
        return t.reshape(n, n, n_head, d).permute(0, 2, 1, 3)

    q = heads(_linear(x, _p(p, "to_query.weight", dtype)))
    k = heads(_linear(x, _p(p, "to_key.weight", dtype)))
    v = heads(_linear(x, _p(p, "to_value.weight", dtype)))
    pm = _pair_mask(tokens, dtype) > 0  # [rows, keys]
    keep = pm[:, None, None, :]
    # rows are independent problems: take them in chunks so the [rows, H, n, n] logits of a
    # large N never exist at once (64 rows at N = 1024: 1 GiB of fp32 logits)
    step = max(1, (1 << 28) // max(1, n_head * n * n))
    o = torch.cat([_masked_softmax_attention(q[r:r + step], k[r:r + step], v[r:r + step], bias[None],
                                             keep[r:r + step]) for r in range(0, n, step)])  # [rows, H, n, d]
    o = o.permute(0, 2, 1, 3).reshape(n, n, hidden)
    o = torch.sigmoid(_linear(x, _p(p, "to_gate.weight", dtype))) * o
    delta = _linear(o, _p(p, "to_out.weight", dtype))
    if not starting:
        delta = delta.transpose(0, 1)
    return z + delta


def transition(x: Tensor, p: Params, *, dtype: torch.dtype = torch.float32) -> Tensor:
    """``x + W_sq(silu(W_a LN(x)) * W_b LN(x))``, residual included.

    ``legacy/primitives.py:20-37`` bound by ``legacy/routing.py:28-30,65-79`` to
    ``legacy/reference/transition.py:28-59``; ``swiglu`` is
    ``modules/dense/diffusion_transformer.py:36-44`` (``transition1`` split by
    ``chunk(2)`` into ``expand_a`` / ``expand_b``, ``legacy/released.py:211-224``).
    """
    x = x.to(dtype)
    y = layer_norm(x, _p(p, "ln_in.weight", dtype), _p(p, "ln_in.bias", dtype))
    a = _linear(y, _p(p, "expand_a.weight", dtype))
    b = _linear(y, _p(p, "expand_b.weight", dtype))
    return x + _linear(torch.nn.functional.silu(a) * b, _p(p, "squeeze.weight", dtype))


def attention_pair_bias(
    s: Tensor,
    z: Tensor,
    tokens: Tensor,
    p: Params,
    *,
    n_head: int = 16,
    gate_bias: float = 0.0,
    extra_pair_bias: Tensor | None = None,
    dtype: torch.dtype = torch.float32,
) -> Tensor:
    """Single-track attention with pair bias, residual included.

    ``legacy/pairformer.py:204-226``: the logits bias is ``W_pb LN(z)`` with the pair
    LayerNorm's weight only (its offset is a per-head constant the converter discards,
    ``legacy/released.py:51-62``), plus ``extra_pair_bias`` on every head; the attention
    is ``legacy/transformer.py:88-133`` (``SelfAttention``, no single conditioning: the
    AdaLN is a plain LayerNorm, the output a gated projection,
    ``modules/dense/diffusion_transformer.py:297-349``) with the token key mask.
    """
    s = s.to(dtype)
    z = z.to(dtype)
    n, c_s = s.shape
    zb = layer_norm(z, _p(p, "ln_pair.weight", dtype), None)
    bias = _linear(zb, _p(p, "to_bias.weight", dtype)).permute(2, 0, 1)  # [H, N, N]
    if extra_pair_bias is not None:
        bias = bias + extra_pair_bias.to(dtype)[None]
    y = layer_norm(s, _p(p, "ln_single.weight", dtype), _p(p, "ln_single.bias", dtype))
    d = c_s // n_head

    def heads(t: Tensor) -> Tensor:
        return t.reshape(n, n_head, d).permute(1, 0, 2)

    q = heads(_linear(y, _p(p, "to_query.weight", dtype), _p(p, "to_query.bias", dtype)))
    k = heads(_linear(y, _p(p, "to_key.weight", dtype)))
    v = heads(_linear(y, _p(p, "to_value.weight", dtype)))
    keep = (tokens > 0)[None, None, :]
    o = _masked_softmax_attention(q, k, v, bias, keep)  # [H, N, d]
    o = o.permute(1, 0, 2).reshape(n, c_s)
    gate = _linear(y, _p(p, "to_gate.weight", dtype))
    if gate_bias:
        gate = gate + gate_bias
    delta = _linear(torch.sigmoid(gate) * o, _p(p, "to_out.weight", dtype))
    return s + delta


def _sub(p: Params, prefix: str) -> dict[str, Tensor]:
    return {k[len(prefix) + 1 :]: v for k, v in p.items() if k.startswith(prefix + ".")}


def pairformer_block(
    z: Tensor,
    s: Tensor | None,
    tokens: Tensor,
    p: Params,
    *,
    n_head_pair: int = 4,
    n_head_single: int = 16,
    gate_bias: float = 0.0,
    extra_pair_bias: Tensor | None = None,
    dtype: torch.dtype = torch.float32,
    storage: torch.dtype | None = None,
) -> tuple[Tensor, Tensor | None]:
    """One sequential (AF3) Pairformer block: ``legacy/pairformer.py:191-229``.

    ``z += TMo; z += TMi; z += TAs; z += TAe; z += Tr(z); s += APB(s, z); s += Tr(s)``.

    ``storage``: the activation dtype between ops. ``None`` keeps ``dtype`` throughout;
    ``torch.bfloat16`` rounds the pair and the single to bf16 after every op, as the
    master-precision activation stream stores them (fp32 parameters and arithmetic, bf16
    activations at the op boundaries, ``modules/engine/configure.py:73-99``).
    """

    def keep(x: Tensor) -> Tensor:
        return x if storage is None else x.to(storage).to(dtype)

    z = keep(triangle_multiplication(z, tokens, _sub(p, "tri_multi_outgoing"), outgoing=True, dtype=dtype))
    z = keep(triangle_multiplication(z, tokens, _sub(p, "tri_multi_incoming"), outgoing=False, dtype=dtype))
    z = keep(triangle_attention(z, tokens, _sub(p, "tri_atten_starting"), starting=True, n_head=n_head_pair,
                                dtype=dtype))
    z = keep(triangle_attention(z, tokens, _sub(p, "tri_atten_ending"), starting=False, n_head=n_head_pair,
                                dtype=dtype))
    z = keep(transition(z, _sub(p, "transition_pair"), dtype=dtype))
    if s is None:
        return z, None
    s = keep(attention_pair_bias(
        s, z, tokens, _sub(p, "single_attention"), n_head=n_head_single, gate_bias=gate_bias,
        extra_pair_bias=extra_pair_bias, dtype=dtype,
    ))
    s = keep(transition(s, _sub(p, "single_transition"), dtype=dtype))
    return z, s


def rel_l2(got: Tensor, want: Tensor, where: Tensor | None = None) -> float:
    """Relative L2 error ``|got - want| / |want|`` in float64, optionally on ``where``."""
    g, w = got.double(), want.double()
    if where is not None:
        g, w = g[where], w[where]
    return (torch.linalg.vector_norm(g - w) / torch.linalg.vector_norm(w).clamp_min(1e-30)).item()


def block_flops(n: int, c: int = 128, c_s: int = 384) -> float:
    """Algorithmic flops of one block (multiply-add = 2), the figure the bench reports against."""
    del c, c_s
    return 1536.0 * n**3 + 1_121_792.0 * n**2 + 5.0e6 * n


__all__ = [
    "MASK_VALUE",
    "attention_pair_bias",
    "block_flops",
    "layer_norm",
    "pairformer_block",
    "rel_l2",
    "transition",
    "triangle_attention",
    "triangle_multiplication",
]
