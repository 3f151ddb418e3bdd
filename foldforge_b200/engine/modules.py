"""The engine op classes of the Pairformer pair stack, with a ``pytorch`` and a ``b200`` backend.

These re-provide the engine-module contract FoldForge's graph consumes (the classes of
``miniworld_engine.modules`` that ``src/foldforge/modules/engine/{modules,pairformer}.py``
build): the same class names, constructor arguments, child names and state-dict keys
(the schema ``legacy/released.py:318-369`` writes), ``backends`` / ``backend`` /
``set_backend`` / ``unsupported`` / ``_forward_<backend>``, the ``dead`` flag and the
``MasterWeights`` mixin. Every op returns its input PLUS its update (the residual is owned).

* ``pytorch``: the reference equations (``legacy/reference/*.py``) on batched tensors, in
  fp32 internally, output in the input dtype.
* ``b200``: the sm_100a kernels through the C ABI (:mod:`foldforge_b200.kernels`); it
  never falls back by itself -- a call outside its range is refused by ``unsupported()``
  and the caller's guard decides (``engine.unsupported``).

Masked positions: ``masked_update = "zero"`` (default) leaves every pair (i, j) with
``mask_i * mask_j == 0`` and every padded single row exactly unchanged; ``"compute"``
applies the reference equations there too.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

Tensor = torch.Tensor
MASKED_UPDATES = ("zero", "compute")


class BackendUnsupported(RuntimeError):
    """A call outside the selected backend's range, made directly (without the guard)."""


class MasterWeights:
    """fp32 master parameters: under ``set_master_weights()`` a bulk cast keeps them fp32
    (the kernels cast to bf16 themselves); LayerNorm affines are fp32 under any cast."""

    master_weights: bool = False

    def set_master_weights(self) -> None:
        for m in self.modules():  # type: ignore[attr-defined]
            if isinstance(m, MasterWeights):
                m.master_weights = True

    def _apply(self, fn, recurse=True):  # noqa: ANN001 - torch.nn.Module._apply signature
        out = super()._apply(fn, recurse)  # type: ignore[misc]
        if self.master_weights:
            for p in self.parameters():  # type: ignore[attr-defined]
                if p.is_floating_point() and p.dtype != torch.float32:
                    p.data = p.data.float()
        return out


class LayerNorm(nn.LayerNorm):
    """The engine ``LayerNorm``: fp32 affine under any cast; backends ``pytorch`` / ``b200``.
    Not a residual module, so it has no ``dead`` flag."""

    backends = ("pytorch", "b200")
    dispatches_policy = True

    def __init__(self, d, eps: float = 1e-5, bias: bool = True, elementwise_affine: bool = True) -> None:
        super().__init__(d, eps=eps, elementwise_affine=elementwise_affine, bias=bias)
        self.backend = "pytorch"

    def _apply(self, fn, recurse=True):  # noqa: ANN001
        out = super()._apply(fn, recurse)
        for p in self.parameters(recurse=False):
            if p.dtype != torch.float32:
                p.data = p.data.float()
        return out

    def set_backend(self, name: str) -> None:
        _check_backend(self, name)
        self.backend = name

    def unsupported(self, x: Tensor) -> str | None:
        if self.backend == "pytorch":
            return None
        reason = _cuda_reason(x)
        if reason:
            return reason
        if x.dtype not in (torch.bfloat16, torch.float32):
            return f"dtype {x.dtype} (bf16 or fp32 only)"
        if len(self.normalized_shape) != 1:
            return "normalisation over more than one axis"
        return None

    def forward(self, x: Tensor) -> Tensor:
        return _dispatch(self, x)

    def _forward_pytorch(self, x: Tensor) -> Tensor:
        w = None if self.weight is None else self.weight.float()
        b = None if self.bias is None else self.bias.float()
        return F.layer_norm(x.float(), self.normalized_shape, w, b, self.eps).to(x.dtype)

    def _forward_b200(self, x: Tensor) -> Tensor:
        from foldforge_b200 import kernels

        return kernels.layer_norm(x, self.weight, self.bias, self.eps)


# --------------------------------------------------------------------------- helpers
def _check_backend(module: nn.Module, name: str) -> None:
    if name not in type(module).backends:
        message = f"{type(module).__name__} has no {name!r} backend (available: {', '.join(type(module).backends)})"
        raise BackendUnsupported(message)


def _cuda_reason(*ts: Tensor | None) -> str | None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            return "tensor is not on a CUDA device"
        if torch.cuda.get_device_capability(t.device) != (10, 0):
            return "the b200 kernels need an sm_100 device"
        if t.requires_grad and torch.is_grad_enabled():
            return "autograd is not supported by the b200 kernels (inference only)"
    return None


def _library_reason() -> str | None:
    from foldforge_b200 import _lib

    try:
        _lib.load()
    except _lib.LibraryMissing as exc:
        return str(exc)
    return None


def _dispatch(module: nn.Module, *args, **kwargs):
    """Run ``module`` on its backend. A call the backend refuses (``unsupported`` gives a
    reason) raises :class:`BackendUnsupported` unless the module is guarded
    (:func:`foldforge_b200.engine.policy.guard`): then its ``engine.unsupported`` policy runs
    the ``pytorch`` backend (one log line) or raises, and the call is counted in the
    observations."""
    backend = module.backend
    guarded = module.__dict__.get("_ffb_guarded", False)
    served = backend
    reason = None if backend == "pytorch" else module.unsupported(*args, **kwargs)
    if reason is not None:
        if not guarded:
            raise BackendUnsupported(f"{type(module).__name__} backend {backend!r}: {reason}")
        from foldforge_b200.engine import policy

        served = policy.fallback_backend(module, backend, *args, **kwargs)
        policy.refuse(module, reason, served)
    if guarded:
        from foldforge_b200.engine.serving import observe_call

        observe_call(module, backend, reason, served)
    return getattr(module, f"_forward_{served}")(*args, **kwargs)


def honours_dead(forward):
    """A residual op's ``_forward_<backend>``: a module flagged ``dead`` returns its residual
    input unchanged when it runs without grad outside training (``modules/dense/dead.py:1-11``),
    whichever caller (this package's dispatch or FoldForge's own guard) invoked the backend."""

    def run(self, x, *args, **kwargs):
        if self.dead and not self.training and not torch.is_grad_enabled():
            return x
        return forward(self, x, *args, **kwargs)

    run.__name__, run.__doc__, run.__wrapped__ = forward.__name__, forward.__doc__, forward
    return run


def _pair_mask(key_mask: Tensor | None, x: Tensor) -> Tensor:
    if key_mask is None:
        return torch.ones(x.shape[:-1], device=x.device, dtype=torch.float32)
    m = key_mask.float()
    return m[:, :, None] * m[:, None, :]


def _linear(x: Tensor, layer: nn.Linear) -> Tensor:
    return F.linear(x, layer.weight.float(), None if layer.bias is None else layer.bias.float())


def _ln(x: Tensor, norm: nn.LayerNorm) -> Tensor:
    w = None if norm.weight is None else norm.weight.float()
    b = None if norm.bias is None else norm.bias.float()
    return F.layer_norm(x, norm.normalized_shape, w, b, norm.eps)


class _PairOp(MasterWeights, nn.Module):
    """Shared plumbing of the pair ops: backend selection, refusals, the packed-weight cache."""

    backends = ("pytorch", "b200")
    dispatches_policy = True
    #: a flagged module returns its residual input unchanged (``honours_dead``)
    dead = False
    #: channels the b200 kernels are built for
    b200_channels = 128

    def __init__(self) -> None:
        super().__init__()
        self.backend = "pytorch"
        self.masked_update = "zero"
        self._packed: tuple[tuple, Tensor] | None = None

    def set_backend(self, name: str) -> None:
        _check_backend(self, name)
        self.backend = name

    def _pair_reason(self, x: Tensor, key_mask: Tensor | None) -> str | None:
        reason = _cuda_reason(x, key_mask) or _library_reason()
        if reason:
            return reason
        if x.dtype not in (torch.bfloat16, torch.float32):
            return f"activations are {x.dtype}; the b200 kernels take bf16 (master) or fp32"
        if x.dim() != 4 or x.shape[1] != x.shape[2]:
            return f"pair tensor shape {tuple(x.shape)} is not [B, N, N, c]"
        if key_mask is not None and tuple(key_mask.shape) != tuple(x.shape[:2]):
            return f"key mask {tuple(key_mask.shape)} does not match pair {tuple(x.shape)}"
        return None

    def _weights(self) -> dict[str, Tensor]:
        return {k: v.detach() for k, v in self.state_dict().items()}

    def _on_generic(self, fn, x: Tensor, *args, **kwargs) -> Tensor:
        """Run ``fn`` (an fp32 SIMT op of ``csrc/generic.cu``) in fp32 and return ``x``'s dtype:
        the fp32 precision, and widths the tcgen05 kernels are not built for."""
        out = fn(x.float(), *args, **kwargs)
        return out if x.dtype == torch.float32 else out.to(x.dtype)

    def _cached_pack(self, pack) -> Tensor:
        """The packed device image of the weights, rebuilt only when a parameter changed
        (its storage or version): ``pack(weights)`` gets the state dict then."""
        key = tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._packed is None or self._packed[0] != key:
            with torch.no_grad():
                self._packed = (key, pack(dict(self.state_dict())))
        return self._packed[1]

    def _key_mask(self, x: Tensor, key_mask: Tensor | None) -> Tensor:
        if key_mask is None:
            return torch.ones(x.shape[:2], dtype=torch.bool, device=x.device)
        return key_mask

    def _masked_zero(self) -> bool:
        if self.masked_update not in MASKED_UPDATES:
            raise ValueError(f"masked_update must be one of {MASKED_UPDATES}, got {self.masked_update!r}")
        return self.masked_update == "zero"

    def _zero_masked(self, x: Tensor, delta: Tensor, key_mask: Tensor | None) -> Tensor:
        if self._masked_zero() and key_mask is not None:
            delta = delta * _pair_mask(key_mask, x)[..., None]
        return (x.float() + delta).to(x.dtype)


# --------------------------------------------------------------------------- triangle multiplication
class TriangleMultiplication(_PairOp):
    """Triangle multiplicative update, outgoing or incoming, residual included.

    Reference equations: ``legacy/reference/triangle.py:19-50`` (``triangle_update``),
    engine left/right per ``legacy/released.py:135-173``.
    """

    def __init__(self, d_pair: int, d_hidden: int | None = None, outgoing: bool = True, p_drop: float = 0.0,
                 model: str | None = None) -> None:
        super().__init__()
        if model not in (None, "af3"):
            raise ValueError(f"TriangleMultiplication(model={model!r}): only the AF3 form is built here")
        hidden = d_hidden or d_pair
        self.d_pair, self.d_hidden, self.outgoing, self.p_drop = d_pair, hidden, outgoing, p_drop
        self.ln_pair = LayerNorm(d_pair)
        self.ln_out = LayerNorm(hidden)
        self.to_left = nn.Linear(d_pair, hidden, bias=False)
        self.to_right = nn.Linear(d_pair, hidden, bias=False)
        self.to_left_gate = nn.Linear(d_pair, hidden, bias=False)
        self.to_right_gate = nn.Linear(d_pair, hidden, bias=False)
        self.to_out = nn.Linear(hidden, d_pair, bias=False)
        self.to_gate = nn.Linear(d_pair, d_pair, bias=False)

    def unsupported(self, x: Tensor, key_mask: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        return self._pair_reason(x, key_mask)

    def _tensor_cores(self, x: Tensor) -> bool:
        """bf16 at the AF3 widths runs the tcgen05 kernels; anything else the fp32 SIMT path."""
        return x.dtype == torch.bfloat16 and x.shape[-1] == 128 and self.d_hidden == 128

    def forward(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        return _dispatch(self, x, key_mask)

    @honours_dead
    def _forward_pytorch(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        z = x.float()
        v = _ln(z, self.ln_pair)
        m = _pair_mask(key_mask, z)[..., None]
        left = _linear(v, self.to_left) * m * torch.sigmoid(_linear(v, self.to_left_gate))
        right = _linear(v, self.to_right) * m * torch.sigmoid(_linear(v, self.to_right_gate))
        eq = "bikc,bjkc->bijc" if self.outgoing else "bkic,bkjc->bijc"
        u = torch.einsum(eq, left, right)
        delta = _linear(_ln(u, self.ln_out), self.to_out) * torch.sigmoid(_linear(v, self.to_gate))
        return self._zero_masked(x, delta, key_mask)

    @honours_dead
    def _forward_b200(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        if not self._tensor_cores(x):
            return self._on_generic(kernels.trimul_f32, x, self._key_mask(x, key_mask), self._weights(),
                                    outgoing=self.outgoing, masked_zero=self._masked_zero())
        packed = self._cached_pack(lambda w: kernels.trimul_prepare(w, x.device))
        return kernels.trimul(x, self._key_mask(x, key_mask), packed, outgoing=self.outgoing,
                              masked_zero=self._masked_zero())


# --------------------------------------------------------------------------- triangle attention
TRIANGLE_ATTENTION_MODELS: dict[str, str] = {"af3": "TriangleAttentionAF3"}


class TriangleAttention(_PairOp):
    """Triangle attention around the starting (rows) or ending (columns) node.

    ``TriangleAttention(..., model=key)`` builds the class of ``key``; only AF3's
    (``TriangleAttentionAF3``: untransposed pair bias, no projection biases) is built here.
    Reference equations: ``legacy/attention.py:108-171``, ``legacy/reference/attention.py:14-100``.
    """

    def __new__(cls, *args, model: str = "af3", **kwargs):  # noqa: D102 - dispatch on the model key
        if cls is TriangleAttention:
            name = TRIANGLE_ATTENTION_MODELS.get(model)
            if name is None:
                raise ValueError(f"TriangleAttention(model={model!r}): known {sorted(TRIANGLE_ATTENTION_MODELS)}")
            cls = globals()[name]
        return super().__new__(cls)

    def __init__(self, d_pair: int, n_head: int, d_hidden: int | None = None, starting: bool = True,
                 p_drop: float = 0.0, model: str = "af3") -> None:
        super().__init__()
        hidden = d_hidden * n_head if d_hidden else d_pair
        self.d_pair, self.n_head, self.starting, self.p_drop, self.model = d_pair, n_head, starting, p_drop, model
        self.d_head = hidden // n_head
        self.ln_pair = LayerNorm(d_pair)
        self.to_bias = nn.Linear(d_pair, n_head, bias=False)
        self.to_query = nn.Linear(d_pair, hidden, bias=False)
        self.to_key = nn.Linear(d_pair, hidden, bias=False)
        self.to_value = nn.Linear(d_pair, hidden, bias=False)
        self.to_gate = nn.Linear(d_pair, hidden, bias=False)
        self.to_out = nn.Linear(hidden, d_pair, bias=False)

    def unsupported(self, x: Tensor, key_mask: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        if self.d_head > 64:
            return f"head width {self.d_head} (the b200 kernels take at most 64)"
        return self._pair_reason(x, key_mask)

    def _tensor_cores(self, x: Tensor) -> bool:
        return x.dtype == torch.bfloat16 and x.shape[-1] == 128 and (self.n_head, self.d_head) == (4, 32)

    def forward(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        return _dispatch(self, x, key_mask)

    @honours_dead
    def _forward_pytorch(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        z = x.float()
        b, n = z.shape[0], z.shape[1]
        v = _ln(z, self.ln_pair)
        bias = _linear(v, self.to_bias).permute(0, 3, 1, 2)  # [B, H, q, k]
        if not self.starting:
            v = v.transpose(1, 2)

        def heads(t: Tensor) -> Tensor:  # [B, rows, n, H*d] -> [B, rows, H, n, d]
            return t.reshape(b, n, n, self.n_head, self.d_head).permute(0, 1, 3, 2, 4)

        q = heads(_linear(v, self.to_query)) * self.d_head**-0.5
        k = heads(_linear(v, self.to_key))
        val = heads(_linear(v, self.to_value))
        logits = q @ k.transpose(-1, -2) + bias[:, None]
        keep = (_pair_mask(key_mask, z) > 0)[:, :, None, None, :]
        logits = logits.masked_fill(~keep, -1e9)
        o = (logits.softmax(-1) @ val).permute(0, 1, 3, 2, 4).reshape(b, n, n, -1)
        delta = _linear(torch.sigmoid(_linear(v, self.to_gate)) * o, self.to_out)
        if not self.starting:
            delta = delta.transpose(1, 2)
        return self._zero_masked(x, delta, key_mask)

    @honours_dead
    def _forward_b200(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        if not self._tensor_cores(x):
            return self._on_generic(kernels.triattn_f32, x, self._key_mask(x, key_mask), self._weights(),
                                    starting=self.starting, n_head=self.n_head, masked_zero=self._masked_zero())
        packed = self._cached_pack(lambda w: kernels.triattn_prepare(w, x.device))
        return kernels.triattn(x, self._key_mask(x, key_mask), packed, starting=self.starting,
                               masked_zero=self._masked_zero())


class TriangleAttentionAF3(TriangleAttention):
    """AF3's triangle attention (``model="af3"``)."""


# --------------------------------------------------------------------------- transition
class Transition(_PairOp):
    """``x + W_sq(silu(W_a LN(x)) * W_b LN(x))`` (``legacy/primitives.py:20-37``,
    ``legacy/reference/transition.py:28-59``). On b200: the pair (128, 4) and single (384, 4)
    widths in bf16 run the tcgen05 kernels, every other width and fp32 the SIMT path."""

    def __init__(self, d_hidden: int, n: int = 4) -> None:
        super().__init__()
        self.d, self.n = d_hidden, n
        self.ln_in = LayerNorm(d_hidden)
        self.expand_a = nn.Linear(d_hidden, n * d_hidden, bias=False)
        self.expand_b = nn.Linear(d_hidden, n * d_hidden, bias=False)
        self.squeeze = nn.Linear(n * d_hidden, d_hidden, bias=False)

    def unsupported(self, x: Tensor, key_mask: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        reason = _cuda_reason(x, key_mask) or _library_reason()
        if reason:
            return reason
        if x.dtype not in (torch.bfloat16, torch.float32):
            return f"activations are {x.dtype}; the b200 kernels take bf16 (master) or fp32"
        if key_mask is None:
            return None if x.dim() >= 2 else f"transition input {tuple(x.shape)} has no rows"
        if x.dim() == 4 and x.shape[1] != x.shape[2] or x.dim() not in (3, 4):
            return f"transition input {tuple(x.shape)} is neither a pair [B, N, N, c] nor a single [B, N, c]"
        if tuple(key_mask.shape) != tuple(x.shape[:2]):
            return f"key mask {tuple(key_mask.shape)} does not match {tuple(x.shape)}"
        return None

    def _tensor_cores(self, x: Tensor) -> bool:
        """The fused AF3-width kernels: the pair transition (128, 4) and the single one (384, 4)."""
        if x.dtype != torch.bfloat16 or self.n != 4:
            return False
        return (self.d == 128 and x.dim() == 4 and x.shape[1] == x.shape[2]) or (self.d == 384 and x.dim() == 3)

    def _gemm_rows(self, x: Tensor, key_mask: Tensor | None) -> bool:
        """Unmasked bf16 rows of other widths (the MSA transition): the tensor-core GEMM transition."""
        return (x.dtype == torch.bfloat16 and key_mask is None and self.d % 8 == 0 and (self.n * self.d) % 16 == 0)

    def forward(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        return _dispatch(self, x, key_mask)

    @honours_dead
    def _forward_pytorch(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        v = _ln(x.float(), self.ln_in)
        delta = _linear(F.silu(_linear(v, self.expand_a)) * _linear(v, self.expand_b), self.squeeze)
        if self._masked_zero() and key_mask is not None:
            m = _pair_mask(key_mask, x) if x.dim() == 4 else key_mask.float()
            delta = delta * m[..., None]
        return (x.float() + delta).to(x.dtype)

    @honours_dead
    def _forward_b200(self, x: Tensor, key_mask: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        if not self._tensor_cores(x):
            if self._gemm_rows(x, key_mask):
                packed = self._cached_pack(lambda w: kernels.transition_gemm_prepare(w, self.d, self.n, x.device))
                return kernels.transition_gemm(x, packed, self.d, self.n)
            if key_mask is None:  # unmasked: the rows of any leading shape
                rows = x.reshape(1, -1, x.shape[-1])
                return self._on_generic(kernels.transition_f32, rows, None, self._weights(),
                                        masked_zero=False).reshape(x.shape)
            return self._on_generic(kernels.transition_f32, x, key_mask, self._weights(),
                                    masked_zero=self._masked_zero())
        if self.d == 128:
            packed = self._cached_pack(lambda w: kernels.transition_prepare(w, x.device))
            return kernels.transition(x, key_mask, packed, masked_zero=self._masked_zero())
        packed = self._cached_pack(lambda w: kernels.single_transition_prepare(w, x.device))
        return kernels.single_transition(x, key_mask, packed, masked_zero=self._masked_zero())


# --------------------------------------------------------------------------- single attention
class AttentionPairBias(_PairOp):
    """Single-track attention with pair bias, residual included
    (``legacy/pairformer.py:204-226``, ``legacy/transformer.py:88-133``)."""

    def __init__(self, d_single: int, d_pair: int, n_head: int = 16, gate_bias: float = 0.0) -> None:
        super().__init__()
        self.d_single, self.d_pair, self.n_head, self.gate_bias = d_single, d_pair, n_head, gate_bias
        self.ln_single = LayerNorm(d_single)
        self.to_query = nn.Linear(d_single, d_single, bias=True)
        self.to_key = nn.Linear(d_single, d_single, bias=False)
        self.to_value = nn.Linear(d_single, d_single, bias=False)
        self.ln_pair = LayerNorm(d_pair, bias=False)
        self.to_bias = nn.Linear(d_pair, n_head, bias=False)
        self.to_gate = nn.Linear(d_single, d_single, bias=False)
        self.to_out = nn.Linear(d_single, d_single, bias=False)

    def unsupported(self, s: Tensor, z: Tensor, key_mask: Tensor | None = None,
                    extra_pair_bias: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        if self.d_single % self.n_head or self.d_single // self.n_head > 64:
            return f"widths ({self.d_single}, {self.n_head} heads): the b200 kernels take head widths up to 64"
        reason = _cuda_reason(s, z, key_mask, extra_pair_bias) or _library_reason()
        if reason:
            return reason
        if s.dtype not in (torch.bfloat16, torch.float32) or z.dtype != s.dtype:
            return f"activations s {s.dtype}, z {z.dtype} (the b200 kernels take both bf16 or both fp32)"
        if s.dim() != 3 or z.dim() != 4 or z.shape[:2] != s.shape[:2] or z.shape[1] != z.shape[2]:
            return f"shapes s {tuple(s.shape)}, z {tuple(z.shape)}"
        return None

    def _tensor_cores(self, s: Tensor) -> bool:
        return s.dtype == torch.bfloat16 and (self.d_single, self.d_pair, self.n_head) == (384, 128, 16)

    def forward(self, s: Tensor, z: Tensor, key_mask: Tensor | None = None,
                extra_pair_bias: Tensor | None = None) -> Tensor:
        return _dispatch(self, s, z, key_mask, extra_pair_bias)

    @honours_dead
    def _forward_pytorch(self, s: Tensor, z: Tensor, key_mask: Tensor | None = None,
                         extra_pair_bias: Tensor | None = None) -> Tensor:
        b, n, cs = s.shape
        d = cs // self.n_head
        bias = _linear(_ln(z.float(), self.ln_pair), self.to_bias).permute(0, 3, 1, 2)
        if extra_pair_bias is not None:
            bias = bias + extra_pair_bias.float()
        y = _ln(s.float(), self.ln_single)

        def heads(t: Tensor) -> Tensor:
            return t.reshape(b, n, self.n_head, d).permute(0, 2, 1, 3)

        q, k, v = heads(_linear(y, self.to_query)), heads(_linear(y, self.to_key)), heads(_linear(y, self.to_value))
        logits = (q * d**-0.5) @ k.transpose(-1, -2) + bias
        if key_mask is not None:
            logits = logits.masked_fill(~key_mask.bool()[:, None, None, :], -1e9)
        o = (logits.softmax(-1) @ v).permute(0, 2, 1, 3).reshape(b, n, cs)
        gate = _linear(y, self.to_gate) + self.gate_bias
        delta = _linear(torch.sigmoid(gate) * o, self.to_out)
        if self._masked_zero() and key_mask is not None:
            delta = delta * key_mask.float()[..., None]
        return (s.float() + delta).to(s.dtype)

    @honours_dead
    def _forward_b200(self, s: Tensor, z: Tensor, key_mask: Tensor | None = None,
                      extra_pair_bias: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        if not self._tensor_cores(s):
            out = kernels.attention_pair_bias_f32(s.float(), z.float(), self._key_mask(s, key_mask), self._weights(),
                                                  n_head=self.n_head, extra_pair_bias=extra_pair_bias,
                                                  gate_bias=self.gate_bias, masked_zero=self._masked_zero())
            return out.to(s.dtype)

        def pack(w: dict[str, Tensor]) -> Tensor:
            if w.get("to_query.bias") is None:
                w["to_query.bias"] = torch.zeros(self.d_single, device=s.device)
            return kernels.apb_prepare(w, s.device)

        packed = self._cached_pack(pack)
        mask = self._key_mask(s, key_mask)
        return kernels.attention_pair_bias(s, z, mask, packed, extra_pair_bias=extra_pair_bias,
                                           gate_bias=self.gate_bias, masked_zero=self._masked_zero())


# --------------------------------------------------------------------------- MSA module
class OuterProductMean(_PairOp):
    """The outer product mean's RAW update (no residual; the MSA-stack block adds it):
    ``delta[i, j] = (W_o vec(sum_s L[s, i] (x) R[s, j]) + b_o) / d(n_ij)`` with ``L = m W_l LN(msa)``,
    ``R = m W_r LN(msa)`` and ``n_ij = sum_s m_si m_sj`` (``legacy/primitives.py:40-136``,
    ``legacy/reference/attention.py:57-74``; engine keys of ``legacy/released.py:227-250``).
    ``count_offset``: ``d(n) = n + count_offset`` (AF3: 1e-3), ``None``: ``max(n, 1)``.
    ``normalize_before_proj``: divide before adding ``b_o`` (the bias-after-norm variants) instead of
    after (AF3). Called as ``opm(msa [B, S, N, c_m], row_mask [B, S, N])``."""

    def __init__(self, d_msa: int, d_pair: int, d_hidden: int = 32, *, normalize_before_proj: bool = True,
                 projection_bias: bool = False, groups: int = 1, product_norm_eps: float = 0.1,
                 count_offset: float | None = None) -> None:
        super().__init__()
        if groups != 1:
            raise ValueError("the grouped (Chai-1) outer product mean is not built here")
        self.d_msa, self.d_pair, self.d_hidden = d_msa, d_pair, d_hidden
        self.normalize_before_proj, self.projection_bias = normalize_before_proj, projection_bias
        self.count_offset, self.product_norm_eps = count_offset, product_norm_eps
        self.ln_msa = LayerNorm(d_msa)
        self.to_left = nn.Linear(d_msa, d_hidden, bias=projection_bias)
        self.to_right = nn.Linear(d_msa, d_hidden, bias=projection_bias)
        self.to_out = nn.Linear(d_hidden * d_hidden, d_pair, bias=True)

    def unsupported(self, msa: Tensor, row_mask: Tensor) -> str | None:
        if self.backend == "pytorch":
            return None
        if (self.d_msa, self.d_pair, self.d_hidden) != (64, 128, 32):
            return f"widths ({self.d_msa}, {self.d_pair}, {self.d_hidden}) (b200: 64, 128, 32)"
        if self.projection_bias or self.normalize_before_proj:
            return "only AF3's form (no projection bias, the output bias before the divide) has b200 kernels"
        reason = _cuda_reason(msa, row_mask) or _library_reason()
        if reason:
            return reason
        if msa.dtype != torch.bfloat16:
            return f"activations are {msa.dtype}; the b200 MSA kernels take bf16 (master precision)"
        if msa.dim() != 4 or tuple(row_mask.shape) != tuple(msa.shape[:3]):
            return f"msa {tuple(msa.shape)} / row mask {tuple(row_mask.shape)} are not [B, S, N, c] / [B, S, N]"
        return None

    def forward(self, msa: Tensor, row_mask: Tensor) -> Tensor:
        return _dispatch(self, msa, row_mask)

    def _forward_pytorch(self, msa: Tensor, row_mask: Tensor) -> Tensor:
        m = row_mask.float()[..., None]
        x = _ln(msa.float(), self.ln_msa)
        left, right = m * _linear(x, self.to_left), m * _linear(x, self.to_right)
        b, _, n, k = left.shape
        outer = torch.einsum("bsic,bsje->bijce", left, right).reshape(b, n, n, k * k)
        count = torch.einsum("bsi,bsj->bij", m[..., 0], m[..., 0])[..., None]
        divisor = count.clamp_min(1.0) if self.count_offset is None else count + self.count_offset
        w = self.to_out.weight.float()
        if self.normalize_before_proj:
            delta = (outer @ w.t()) / divisor + self.to_out.bias.float()
        else:
            delta = (outer @ w.t() + self.to_out.bias.float()) / divisor
        return delta.to(msa.dtype)

    def _forward_b200(self, msa: Tensor, row_mask: Tensor) -> Tensor:
        from foldforge_b200 import kernels

        packed = self._cached_pack(lambda w: kernels.opm_prepare(w, msa.device))
        return kernels.outer_product_mean(msa, row_mask, packed, count_offset=self.count_offset)


class MSAPairWeightedAveraging(_PairOp):
    """MSA pair-weighted averaging with residual: per head, the pair's logits ``W_b LN(z)[i, j]``
    (minus 1e9 at columns no MSA row has) give softmax weights over j that average the values
    ``W_v LN(msa)`` of each MSA row; sigmoid-gated by ``W_g LN(msa)``, projected back by ``W_o``
    (``legacy/attention.py:174-229``; engine keys of ``legacy/released.py:253-281``). Called as
    ``pwa(msa [B, S, N, c_m], pair [B, N, N, c_z], key_mask [B, N])``."""

    def __init__(self, d_msa: int, d_pair: int, n_head: int = 8, d_hidden: int | None = None,
                 p_drop: float = 0.0) -> None:
        super().__init__()
        self.d_msa, self.d_pair, self.n_head, self.p_drop = d_msa, d_pair, n_head, p_drop
        self.d_hidden = d_hidden or d_msa // n_head
        hidden = n_head * self.d_hidden
        self.ln_msa = LayerNorm(d_msa)
        self.ln_pair = LayerNorm(d_pair, bias=False)
        self.to_bias = nn.Linear(d_pair, n_head, bias=False)
        self.to_value = nn.Linear(d_msa, hidden, bias=False)
        self.to_gate = nn.Linear(d_msa, hidden, bias=False)
        self.to_out = nn.Linear(hidden, d_msa, bias=False)

    def unsupported(self, msa: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        if (self.d_msa, self.d_pair, self.n_head, self.d_hidden) != (64, 128, 8, 8):
            return f"widths ({self.d_msa}, {self.d_pair}, {self.n_head} x {self.d_hidden}) (b200: 64, 128, 8 x 8)"
        reason = _cuda_reason(msa, pair, key_mask) or _library_reason()
        if reason:
            return reason
        if msa.dtype != torch.bfloat16 or pair.dtype != torch.bfloat16:
            return "activations must be bf16 (master precision)"
        if msa.dim() != 4 or pair.dim() != 4 or pair.shape[:2] != (msa.shape[0], msa.shape[2]):
            return f"shapes msa {tuple(msa.shape)}, pair {tuple(pair.shape)}"
        return None

    def forward(self, msa: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        return _dispatch(self, msa, pair, key_mask)

    @honours_dead
    def _forward_pytorch(self, msa: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        x = _ln(msa.float(), self.ln_msa)
        logits = _linear(_ln(pair.float(), self.ln_pair), self.to_bias).permute(0, 3, 1, 2)  # [B, H, i, j]
        if key_mask is not None:
            logits = logits + 1e9 * (key_mask.float()[:, None, None, :] - 1.0)
        weights = torch.softmax(logits, dim=-1)
        b, s, n, _ = x.shape
        v = _linear(x, self.to_value).reshape(b, s, n, self.n_head, self.d_hidden)
        avg = torch.einsum("bhij,bsjhc->bsihc", weights, v).reshape(b, s, n, -1)
        delta = _linear(torch.sigmoid(_linear(x, self.to_gate)) * avg, self.to_out)
        return (msa.float() + delta).to(msa.dtype)

    @honours_dead
    def _forward_b200(self, msa: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        packed = self._cached_pack(lambda w: kernels.pwa_prepare(w, msa.device))
        if key_mask is None:
            key_mask = torch.ones(pair.shape[:2], dtype=torch.bool, device=pair.device)
        return kernels.pair_weighted_averaging(msa, pair, key_mask, packed)


# --------------------------------------------------------------------------- the block
@dataclass(frozen=True)
class PairformerConfig:
    """The engine block's configuration (``modules/engine/pairformer.py:38-53``)."""

    d_pair: int = 128
    d_hidden_tri_multi: int = 128
    d_hidden_tri_attention: int = 32
    n_head_tri_attention: int = 4
    p_drop: float = 0.0
    use_triangle_attention: bool = True
    model: str = "af3"
    d_single: int = 384
    n_head_single: int = 16
    single_gate_bias: float = 0.0
    pair_transition_n: int = 4
    single_transition_n: int = 4
    parallel: bool = False
    masked_update: str = "zero"


class PairformerBlock(MasterWeights, nn.Module):
    """One AF3 Pairformer block (``legacy/pairformer.py:191-229``, sequential schedule):
    ``z += TMo; z += TMi; z += TAs; z += TAe; z += Tr(z); s += APB(s, z); s += Tr(s)``.

    Called as ``block(pair [B, N, N, c], key_mask [B, N] bool, single [B, N, c_s] = None,
    extra_pair_bias [B, H_s, N, N] = None)``; returns ``pair`` or ``(pair, single)``.
    """

    backends = ("pytorch", "b200")

    def __init__(self, config: PairformerConfig) -> None:
        super().__init__()
        if config.parallel:
            raise ValueError("the parallel (Chai-1 / RoseTTAFold3) schedule is not built here")
        if config.masked_update not in MASKED_UPDATES:
            raise ValueError(f"masked_update must be one of {MASKED_UPDATES}")
        self.config = config
        self.backend = "pytorch"
        c = config.d_pair
        self.tri_multi_outgoing = TriangleMultiplication(c, config.d_hidden_tri_multi, outgoing=True)
        self.tri_multi_incoming = TriangleMultiplication(c, config.d_hidden_tri_multi, outgoing=False)
        if config.use_triangle_attention:
            self.tri_atten_starting = TriangleAttention(c, config.n_head_tri_attention,
                                                        d_hidden=config.d_hidden_tri_attention, starting=True,
                                                        model=config.model)
            self.tri_atten_ending = TriangleAttention(c, config.n_head_tri_attention,
                                                      d_hidden=config.d_hidden_tri_attention, starting=False,
                                                      model=config.model)
        self.transition_pair = Transition(c, config.pair_transition_n)
        if config.d_single > 0:
            self.single_attention = AttentionPairBias(config.d_single, c, config.n_head_single,
                                                      config.single_gate_bias)
            self.single_transition = Transition(config.d_single, config.single_transition_n)
        for m in self.modules():
            if isinstance(m, _PairOp):
                m.masked_update = config.masked_update

    def set_backend(self, name: str) -> None:
        """Put every child op on ``name`` (the composite itself stays a plain module)."""
        _check_backend(self, name)
        for m in self.modules():
            if isinstance(m, _PairOp):
                m.set_backend(name)

    def forward(self, pair: Tensor, key_mask: Tensor | None = None, single: Tensor | None = None,
                extra_pair_bias: Tensor | None = None):
        pair = self.tri_multi_outgoing(pair, key_mask)
        pair = self.tri_multi_incoming(pair, key_mask)
        if self.config.use_triangle_attention:
            pair = self.tri_atten_starting(pair, key_mask)
            pair = self.tri_atten_ending(pair, key_mask)
        pair = self.transition_pair(pair, key_mask)
        if single is None or self.config.d_single <= 0:
            return pair
        single = self.single_attention(single, pair, key_mask, extra_pair_bias)
        single = self.single_transition(single, key_mask)
        return pair, single


class Pairformer(MasterWeights, nn.Module):
    """A stack of :class:`PairformerBlock` (the trunk), run in order."""

    backends = ("pytorch", "b200")

    def __init__(self, config: PairformerConfig, n_blocks: int) -> None:
        super().__init__()
        self.config = config
        self.backend = "pytorch"
        self.blocks = nn.ModuleList(PairformerBlock(config) for _ in range(n_blocks))

    def set_backend(self, name: str) -> None:
        _check_backend(self, name)
        for block in self.blocks:
            block.set_backend(name)

    def forward(self, pair: Tensor, key_mask: Tensor | None = None, single: Tensor | None = None,
                extra_pair_bias: Tensor | None = None):
        for block in self.blocks:
            out = block(pair, key_mask, single, extra_pair_bias)
            if single is None:
                pair = out
            else:
                pair, single = out
        return pair if single is None else (pair, single)
