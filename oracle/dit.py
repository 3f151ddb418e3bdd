"""CPU oracle of AF3's token diffusion transformer block (TEST INFRASTRUCTURE ONLY).

Restates, in plain fp32 PyTorch on the ENGINE key schema the converter writes
(``legacy/released.py:372-509``), the released ``DiffusionTransformer`` block with AF3's spec
(``legacy/transformer.py:136-294`` with ``SelfAttention`` :28-135 and
``modules/dense/diffusion_transformer.py``): sigmoid-form adaptive LayerNorm with a
weight-only conditioning norm (:47-89, :180-251), attention with the block's pair logits and
a gated query (``dot_product_attention``: masked logits REPLACED by -1e9 after the bias,
``legacy/reference/attention.py:14-54``), the AdaLN-Zero output gate on the raw conditioning
(:253-350), the SwiGLU transition (:133-149, :353-404), and one residual after each
(``conditioned_residual`` :92-104). Who may use it: ``tests/`` and ``bench.py``'s CPU legs,
as the checker.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle.pairformer import LN_EPS, _sub, layer_norm

Tensor = torch.Tensor


def adaptive_layer_norm(x: Tensor, cond: Tensor, p: dict[str, Tensor]) -> Tensor:
    """``sigmoid(W_s LN_c(cond) + b_s) * LN(x) + W_b LN_c(cond)``: LN(x) without an affine, the
    conditioning norm with a weight only."""
    value = F.layer_norm(x, (x.shape[-1],), eps=LN_EPS)
    ctx = layer_norm(cond, p["ln_cond.weight"], None)
    return torch.sigmoid(ctx @ p["to_scale.weight"].t() + p["to_scale.bias"]) * value + ctx @ p["to_bias.weight"].t()


def pair_logits(pair: Tensor, p: dict[str, Tensor]) -> Tensor:
    """The block's pair bias ``[H, N, N]``: ``W_b LN(pair)`` (the norm's offset, a per-head
    constant the softmax cancels, is not part of the engine block)."""
    return (layer_norm(pair, p["ln_pair.weight"], None) @ p["to_bias.weight"].t()).permute(2, 0, 1)


def attention(x: Tensor, cond: Tensor, logits_bias: Tensor, mask: Tensor, p: dict[str, Tensor], *,
              n_head: int = 16) -> Tensor:
    """The attention delta of a block: ``sigmoid(W_z cond + b_z) * W_o(sigmoid(W_g a) * o)``,
    ``a`` the adaptive-normalised ``x``, ``o`` the pair-biased attention over the tokens."""
    a = adaptive_layer_norm(x, cond, _sub(p, "ada_ln_in"))
    *lead, n, c = a.shape
    d = c // n_head

    def heads(t: Tensor) -> Tensor:
        return t.reshape(*lead, n, n_head, d).transpose(-2, -3)  # [..., H, N, d]

    q = heads(a @ p["to_query.weight"].t() + p["to_query.bias"])
    k = heads(a @ p["to_key.weight"].t())
    v = heads(a @ p["to_value.weight"].t())
    logits = (q * d ** -0.5) @ k.transpose(-1, -2) + logits_bias
    logits = logits.masked_fill(mask.float().reshape(*([1] * (logits.dim() - 1)), n) <= 0, -1e9)
    o = (logits.softmax(-1) @ v).transpose(-2, -3).reshape(*lead, n, c)
    gated = torch.sigmoid(a @ p["to_gate.weight"].t()) * o
    return torch.sigmoid(cond @ p["to_scale.weight"].t() + p["to_scale.bias"]) * (gated @ p["to_out.weight"].t())


def transition(x: Tensor, cond: Tensor, p: dict[str, Tensor]) -> Tensor:
    """The transition delta: ``sigmoid(W_z cond + b_z) * W_sq(silu(W_a a) * W_b a)``."""
    a = adaptive_layer_norm(x, cond, _sub(p, "ada_ln_in"))
    h = F.silu(a @ p["expand_a.weight"].t()) * (a @ p["expand_b.weight"].t())
    return torch.sigmoid(cond @ p["to_scale.weight"].t() + p["to_scale.bias"]) * (h @ p["squeeze.weight"].t())


def token_dit_block(x: Tensor, cond: Tensor, pair: Tensor, mask: Tensor, p: dict[str, Tensor], *,
                    n_head: int = 16) -> Tensor:
    """One block: ``x += attention(x)``, then ``x += transition(x)``; ``x`` ``[..., N, c]``,
    ``cond`` ``[N, c_cond]``, ``pair`` ``[N, N, c_pair]``, ``mask`` ``[N]``."""
    x, cond, pair = x.float(), cond.float(), pair.float()
    bias = pair_logits(pair, _sub(p, "attention"))
    x = x + attention(x, cond, bias, mask, _sub(p, "attention"), n_head=n_head)
    return x + transition(x, cond, _sub(p, "transition"))


def token_dit_stack(x: Tensor, cond: Tensor, pair: Tensor, mask: Tensor, blocks: list[dict[str, Tensor]], *,
                    n_head: int = 16) -> Tensor:
    """The blocks in order."""
    for p in blocks:
        x = token_dit_block(x, cond, pair, mask, p, n_head=n_head)
    return x


__all__ = ["adaptive_layer_norm", "attention", "pair_logits", "token_dit_block", "token_dit_stack", "transition"]
