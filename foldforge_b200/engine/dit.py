"""AF3's token diffusion transformer: the engine ``TokenDiT`` block and FoldForge's stack.

The engine owns one block class per model (``src/foldforge/modules/engine/transformers.py:1-10``);
its state-dict keys are the converter's (``legacy/released.py:372-509``):
``attention.{ada_ln_in.*, to_query, to_key, to_value, to_gate, to_scale, to_out, ln_pair,
to_bias}`` and ``transition.{ada_ln_in.*, expand_a, expand_b, squeeze, to_scale}``. The
algorithm is the released ``DiffusionTransformer`` block with AF3's spec
(``legacy/transformer.py:28-294``): an adaptive LayerNorm from the single conditioning, the
pair-biased attention with a gated query, an AdaLN-Zero output gate on the raw conditioning,
the SwiGLU transition, a residual after each.

:class:`TokenDiTStack` is the reference stack's call (``transformers.py:31-78``): ``act [S, L,
768]`` (or ``[L, 768]``), ``mask [L]``, ``single_cond [L, 384]``, ``pair_cond [L, L, 128]``.
On the ``b200`` backend everything that reads only the conditioning (two AdaLN tables, two
output gates, the pair logits) is computed once per conditioning (the tables are kept with
the conditioning tensors' identity and version, as the engine hoists its pair bias once per
pair object) and a sampler step runs the block's kernels on the activations alone.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from foldforge_b200.engine.modules import (
    MasterWeights,
    _check_backend,
    _cuda_reason,
    _dispatch,
    _library_reason,
)

Tensor = torch.Tensor
#: the widths the b200 kernels are built for: (token, conditioning, pair, heads, transition factor)
B200_WIDTHS = (768, 384, 128, 16, 2)


class AdaptiveLayerNorm(nn.Module):
    """``sigmoid(to_scale(ln_cond(c))) * LN(x) + to_bias(ln_cond(c))``: ``LN(x)`` without an
    affine, the conditioning norm with a weight only (``modules/dense/diffusion_transformer.py:47-89``)."""

    def __init__(self, c: int, c_cond: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.eps = eps
        self.ln_cond = nn.LayerNorm(c_cond, eps=eps, bias=False)
        self.to_scale = nn.Linear(c_cond, c, bias=True)
        self.to_bias = nn.Linear(c_cond, c, bias=False)

    def forward(self, x: Tensor, cond: Tensor) -> Tensor:
        ctx = F.layer_norm(cond.float(), cond.shape[-1:], self.ln_cond.weight.float(), None, self.eps)
        value = F.layer_norm(x.float(), x.shape[-1:], eps=self.eps)
        scale = F.linear(ctx, self.to_scale.weight.float(), self.to_scale.bias.float())
        return torch.sigmoid(scale) * value + F.linear(ctx, self.to_bias.weight.float())


class DiTAttention(nn.Module):
    """Attention with the block's pair bias and a gated query, AdaLN in and AdaLN-Zero out."""

    def __init__(self, c: int, c_cond: int, c_pair: int, n_head: int) -> None:
        super().__init__()
        self.n_head = n_head
        self.ada_ln_in = AdaptiveLayerNorm(c, c_cond)
        self.to_query = nn.Linear(c, c, bias=True)
        self.to_key = nn.Linear(c, c, bias=False)
        self.to_value = nn.Linear(c, c, bias=False)
        self.to_gate = nn.Linear(c, c, bias=False)
        self.to_scale = nn.Linear(c_cond, c, bias=True)
        self.to_out = nn.Linear(c, c, bias=False)
        self.ln_pair = nn.LayerNorm(c_pair, bias=False)
        self.to_bias = nn.Linear(c_pair, n_head, bias=False)

    def pair_logits(self, pair: Tensor) -> Tensor:
        """``[..., H, L, L]`` from ``pair [..., L, L, c_pair]``."""
        z = F.layer_norm(pair.float(), pair.shape[-1:], self.ln_pair.weight.float(), None, self.ln_pair.eps)
        return F.linear(z, self.to_bias.weight.float()).movedim(-1, -3)

    def forward(self, x: Tensor, cond: Tensor, logits: Tensor, key_mask: Tensor) -> Tensor:
        """The attention DELTA. ``x [A, B, L, c]``, ``cond [A, B, L, c_cond]``, ``logits
        [B, H, L, L]``, ``key_mask [B, L]``."""
        a = self.ada_ln_in(x, cond)
        *lead, n, c = a.shape
        d = c // self.n_head

        def heads(t: Tensor) -> Tensor:
            return t.reshape(*lead, n, self.n_head, d).transpose(-2, -3)

        lin = lambda layer: F.linear(a, layer.weight.float(), None if layer.bias is None else layer.bias.float())  # noqa: E731
        q, k, v = heads(lin(self.to_query)), heads(lin(self.to_key)), heads(lin(self.to_value))
        att = (q * d**-0.5) @ k.transpose(-1, -2) + logits
        att = att.masked_fill(~key_mask.bool()[..., None, None, :], -1e9)
        o = (att.softmax(-1) @ v).transpose(-2, -3).reshape(*lead, n, c)
        gated = torch.sigmoid(lin(self.to_gate)) * o
        gate = torch.sigmoid(F.linear(cond.float(), self.to_scale.weight.float(), self.to_scale.bias.float()))
        return gate * F.linear(gated, self.to_out.weight.float())


class ConditionedTransition(nn.Module):
    """``sigmoid(to_scale(c)) * squeeze(silu(expand_a(a)) * expand_b(a))``, ``a`` the AdaLN of x."""

    def __init__(self, c: int, c_cond: int, factor: int = 2) -> None:
        super().__init__()
        self.ada_ln_in = AdaptiveLayerNorm(c, c_cond)
        self.expand_a = nn.Linear(c, factor * c, bias=False)
        self.expand_b = nn.Linear(c, factor * c, bias=False)
        self.squeeze = nn.Linear(factor * c, c, bias=False)
        self.to_scale = nn.Linear(c_cond, c, bias=True)

    def forward(self, x: Tensor, cond: Tensor) -> Tensor:
        """The transition DELTA."""
        a = self.ada_ln_in(x, cond)
        h = F.silu(F.linear(a, self.expand_a.weight.float())) * F.linear(a, self.expand_b.weight.float())
        gate = torch.sigmoid(F.linear(cond.float(), self.to_scale.weight.float(), self.to_scale.bias.float()))
        return gate * F.linear(h, self.squeeze.weight.float())


class TokenDiT(MasterWeights, nn.Module):
    """One AF3 token DiT block (residuals included). ``forward(x [A, B, L, c], cond [A, B, L,
    c_cond], pair [B, L, L, c_pair], key_mask [B, L])``."""

    backends = ("pytorch", "b200")
    dispatches_policy = True

    def __init__(self, c: int = 768, c_cond: int = 384, c_pair: int = 128, n_head: int = 16, factor: int = 2) -> None:
        super().__init__()
        self.widths = (c, c_cond, c_pair, n_head, factor)
        self.attention = DiTAttention(c, c_cond, c_pair, n_head)
        self.transition = ConditionedTransition(c, c_cond, factor)
        self.backend = "pytorch"
        self._packed: tuple | None = None
        self._tables: tuple | None = None

    def set_backend(self, name: str) -> None:
        _check_backend(self, name)
        self.backend = name

    def unsupported(self, x: Tensor, cond: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> str | None:
        if self.backend == "pytorch":
            return None
        if self.widths != B200_WIDTHS:
            return f"widths {self.widths}: the b200 kernels are built for {B200_WIDTHS}"
        reason = _cuda_reason(x, cond, pair, key_mask) or _library_reason()
        if reason:
            return reason
        if x.dtype != torch.bfloat16 or cond.dtype != torch.bfloat16 or pair.dtype != torch.bfloat16:
            return f"activations {x.dtype} / {cond.dtype} / {pair.dtype}: the b200 token DiT takes bf16"
        if x.dim() != 4 or pair.dim() != 4 or pair.shape[0] != 1 or x.shape[1] != 1:
            return f"shapes x {tuple(x.shape)}, pair {tuple(pair.shape)}: the b200 token DiT takes one batch entry"
        if cond.shape[0] > 1 and cond.stride(0) != 0:
            return "the b200 token DiT takes one conditioning shared by the samples (an expanded [L, c_cond])"
        return None

    def forward(self, x: Tensor, cond: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        return _dispatch(self, x, cond, pair, key_mask)

    def _forward_pytorch(self, x: Tensor, cond: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        if key_mask is None:
            key_mask = torch.ones(pair.shape[:2], dtype=torch.bool, device=pair.device)
        logits = self.attention.pair_logits(pair)
        y = x.float() + self.attention(x, cond, logits, key_mask)
        y = y + self.transition(y, cond)
        return y.to(x.dtype)

    def _weights(self) -> dict[str, Tensor]:
        return {k: v.detach() for k, v in self.state_dict().items()}

    def _pack(self, device: torch.device) -> Tensor:
        from foldforge_b200 import kernels

        key = tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._packed is None or self._packed[0] != key:
            with torch.no_grad():
                self._packed = (key, kernels.dit_prepare(self._weights(), device))
        return self._packed[1]

    def _conditioning(self, cond: Tensor, pair: Tensor, packed: Tensor) -> Tensor:
        """The per-fold tables, recomputed only when the conditioning tensors (identity or
        in-place version) or the weights change."""
        from foldforge_b200 import kernels

        key = (cond.data_ptr(), cond._version, tuple(cond.shape), pair.data_ptr(), pair._version, id(packed))
        if self._tables is None or self._tables[0] != key:
            self._tables = (key, kernels.dit_condition(cond.contiguous(), pair.contiguous(), packed))
        return self._tables[1]

    def release_fold(self) -> None:
        """Drop the kept per-fold tables."""
        self._tables = None

    def _forward_b200(self, x: Tensor, cond: Tensor, pair: Tensor, key_mask: Tensor | None = None) -> Tensor:
        from foldforge_b200 import kernels

        a, _, n, c = x.shape
        packed = self._pack(x.device)
        tables = self._conditioning(cond[0, 0], pair[0], packed)
        mask = key_mask[0] if key_mask is not None else torch.ones(n, dtype=torch.bool, device=x.device)
        return kernels.dit_forward(x.reshape(a, n, c), mask, packed, tables).reshape(x.shape)


class TokenDiTStack(nn.Module):
    """``blocks``: the token DiT blocks in order (state-dict keys ``blocks.{i}.<engine names>``),
    called like the reference stack (``transformers.py:31-78``)."""

    def __init__(self, blocks: list[TokenDiT]) -> None:
        super().__init__()
        self.blocks = nn.ModuleList(blocks)

    def forward(self, act: Tensor, mask: Tensor, single_cond: Tensor, pair_cond: Tensor,
                extra_pair_bias: Tensor | None = None, key_mask: Tensor | None = None) -> Tensor:
        if extra_pair_bias is not None:
            raise NotImplementedError("extra_pair_bias (OpenDDE's) is not part of AF3's token transformer")
        if key_mask is None:
            key_mask = (mask > 0)[None]
        unbatched = act.dim() == 2
        x = act[None, None] if unbatched else act[:, None]
        cond = single_cond.expand(*x.shape[:-1], single_cond.shape[-1]) if single_cond.dim() == 2 else single_cond[:, None]
        dtype = x.dtype
        pair = pair_cond[None]
        for block in self.blocks:
            x = block(x, cond, pair, key_mask)
        x = x[0, 0] if unbatched else x[:, 0]
        return x.to(dtype)

    def release_fold(self) -> None:
        for block in self.blocks:
            block.release_fold()
