"""CPU oracle of AF3's MSA-stack block (TEST INFRASTRUCTURE ONLY).

Restates, in plain fp32 PyTorch, the reference's released-layout ``EvoformerBlock``
(``legacy/pairformer.py:233-356``) with AF3's settings (``modules/dense/spec.py:535``:
``msa_update_before_opm=False``, one OPM group of 32 channels, no projection bias, the bias
added before the divide, ``msa_value_dim=None`` so 8 heads of 64 / 8, sequential schedule).
Parameters use the ENGINE key schema the converter writes (``legacy/released.py:227-281,
722-749``). Who may use it: ``tests/`` and ``bench.py``'s CPU legs, as the checker.
"""

from __future__ import annotations

import torch

from oracle.pairformer import (
    LN_EPS,
    _sub,
    layer_norm,
    transition,
    triangle_attention,
    triangle_multiplication,
)

Tensor = torch.Tensor
OPM_COUNT_OFFSET = 1e-3  # legacy/primitives.py:68 (``self.epsilon``)


def outer_product_mean(msa: Tensor, msa_mask: Tensor, p: dict[str, Tensor], *, offset: float = OPM_COUNT_OFFSET) -> Tensor:
    """The raw update ``[N, N, c_z]`` of ``af3_outer_product_mean`` (``legacy/reference/attention.py:57-74``)
    after ``OuterProductMean.forward`` (``legacy/primitives.py:86-103``): LayerNorm, masked left
    and right projections, the outer product summed over MSA rows, the output projection plus
    bias, divided by ``offset + sum_s m_si m_sj``. ``to_out.weight`` is ``[c_z, K K]`` with
    column ``c K + e`` (``legacy/released.py:243``)."""
    msa = msa.float()
    mask = msa_mask.float()[..., None]  # [S, N, 1]
    x = layer_norm(msa, p["ln_msa.weight"].float(), p["ln_msa.bias"].float())
    left = mask * (x @ p["to_left.weight"].float().t())    # [S, N, K]
    right = mask * (x @ p["to_right.weight"].float().t())  # [S, N, K]
    k = left.shape[-1]
    outer = torch.einsum("sic,sje->ijce", left, right).reshape(left.shape[1], right.shape[1], k * k)
    out = outer @ p["to_out.weight"].float().t() + p["to_out.bias"].float()
    norm = torch.einsum("si,sj->ij", mask[..., 0], mask[..., 0])[..., None]
    return out / (offset + norm)


def pair_weighted_averaging(msa: Tensor, msa_mask: Tensor, pair: Tensor, p: dict[str, Tensor], *, n_head: int = 8) -> Tensor:
    """``msa + MSAAttention(msa, msa_mask, pair)`` (``legacy/attention.py:198-229``): per head,
    weights ``softmax_j(W_b LN_z(z)[i, j] + 1e9 (max_s m_sj - 1))`` average the values of the
    MSA row over j; sigmoid-gated, projected back, residual. The pair LayerNorm has no offset
    in the engine schema (a per-head constant, ``legacy/released.py:261-263``)."""
    msa, pair = msa.float(), pair.float()
    x = layer_norm(msa, p["ln_msa.weight"].float(), p["ln_msa.bias"].float())
    zl = layer_norm(pair, p["ln_pair.weight"].float(), None)
    logits = (zl @ p["to_bias.weight"].float().t()).permute(2, 0, 1)  # [H, i, j]
    logits = logits + 1e9 * (torch.max(msa_mask.float(), dim=0).values - 1.0)
    weights = torch.softmax(logits, dim=-1)
    v = x @ p["to_value.weight"].float().t()  # [S, N, H d]
    s_, n, hd = v.shape
    v = v.reshape(s_, n, n_head, hd // n_head)
    avg = torch.einsum("hij,sjhc->sihc", weights, v).reshape(s_, n, hd)
    gate = torch.sigmoid(x @ p["to_gate.weight"].float().t())
    return msa + (gate * avg) @ p["to_out.weight"].float().t()


def evoformer_block(msa: Tensor, pair: Tensor, msa_mask: Tensor, tokens: Tensor, p: dict[str, Tensor], *,
                    n_head_pair: int = 4, storage: torch.dtype | None = None) -> tuple[Tensor, Tensor]:
    """One AF3 MSA-stack block (``legacy/pairformer.py:294-356`` with ``msa_pair_update``,
    ``legacy/reference/composition.py:24-40``, order ``opm_first``): ``z += OPM(m)``;
    ``m = PWA(m, z)``; ``m = m + Tr(m)``; then the pair track ``TMo, TMi, TAs, TAe, Tr`` (the
    pair transition unmasked). ``storage`` rounds the MSA and the pair to that dtype after every
    op, as a bf16 activation stream stores them."""

    def keep(x: Tensor) -> Tensor:
        return x if storage is None else x.to(storage).float()

    msa, pair = msa.float(), pair.float()
    pair = keep(pair + outer_product_mean(msa, msa_mask, _sub(p, "outer_product_mean")))
    msa = keep(pair_weighted_averaging(msa, msa_mask, pair, _sub(p, "msa_attention1")))
    msa = keep(transition(msa, _sub(p, "msa_transition")))
    pair = keep(triangle_multiplication(pair, tokens, _sub(p, "triangle_multiplication_outgoing"), outgoing=True))
    pair = keep(triangle_multiplication(pair, tokens, _sub(p, "triangle_multiplication_incoming"), outgoing=False))
    pair = keep(triangle_attention(pair, tokens, _sub(p, "pair_attention1"), starting=True, n_head=n_head_pair))
    pair = keep(triangle_attention(pair, tokens, _sub(p, "pair_attention2"), starting=False, n_head=n_head_pair))
    pair = keep(transition(pair, _sub(p, "pair_transition")))
    return msa, pair


__all__ = ["LN_EPS", "OPM_COUNT_OFFSET", "evoformer_block", "outer_product_mean", "pair_weighted_averaging"]
