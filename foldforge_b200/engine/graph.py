"""FoldForge's unbatched graph layout around a batched engine block (``src/foldforge/modules/engine/graph.py:191-235``)."""

from __future__ import annotations

import torch
from torch import nn

from foldforge_b200.engine import factories
from foldforge_b200.engine.configure import engine_activation


def run_block(block: nn.Module, pair: torch.Tensor, pair_mask: torch.Tensor, single: torch.Tensor | None = None,
              seq_mask: torch.Tensor | None = None, extra_pair_bias: torch.Tensor | None = None):
    """One pairformer block on FoldForge's layout: ``pair [L, L, d]`` (or ``[S, L, L, d]``),
    ``pair_mask [L, L]``, ``single [L, d]``, ``seq_mask [L]``, ``extra_pair_bias [L, L]`` (added to
    every head of the single attention). Returns ``pair`` or ``(pair, single)`` in the given layout."""
    pair, single = engine_activation(pair), engine_activation(single)
    batched = pair.ndim == 4
    if not batched:
        pair = pair[None]
        single = None if single is None else single[None]
    count = pair.shape[0]
    key_mask = (seq_mask > 0)[None] if seq_mask is not None else factories.residue_mask(pair_mask)
    if count > 1:
        key_mask = key_mask.expand(count, -1).contiguous()
    bias = None
    if extra_pair_bias is not None:
        heads = block.config.n_head_single
        bias = extra_pair_bias.to(pair.dtype)[None, None].expand(count, heads, -1, -1)
    if single is None:
        out = block(pair, key_mask)
        return out if batched else out[0]
    pair, single = block(pair, key_mask, single, bias) if bias is not None else block(pair, key_mask, single)
    return (pair, single) if batched else (pair[0], single[0])
