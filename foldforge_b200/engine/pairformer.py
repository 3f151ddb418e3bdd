"""The engine ``PairformerBlock`` as FoldForge builds it (``src/foldforge/modules/engine/pairformer.py:16-62``)."""

from __future__ import annotations

from foldforge_b200.engine.factories import Precision, finish
from foldforge_b200.engine.modules import PairformerBlock, PairformerConfig


def pairformer_block(
    *,
    d_pair: int,
    triangle_model: str,
    d_single: int = 0,
    d_hidden_tri_multi: int | None = None,
    d_hidden_tri_attention: int = 32,
    n_head_tri_attention: int = 4,
    n_head_single: int = 16,
    single_gate_bias: float = 0.0,
    pair_transition_n: int = 4,
    single_transition_n: int = 4,
    use_triangle_attention: bool = True,
    parallel: bool = False,
    divide_by_length: bool = False,
    precision: Precision = "master",
    norm_eps: float | None = None,
    masked_update: str = "zero",
) -> PairformerBlock:
    """One block (residuals included); ``d_single > 0`` adds the single track."""
    if divide_by_length:
        raise ValueError("the length-divided (RoseTTAFold3 exact) triangle multiplication is not built here")
    config = PairformerConfig(
        d_pair=d_pair,
        d_hidden_tri_multi=d_pair if d_hidden_tri_multi is None else d_hidden_tri_multi,
        d_hidden_tri_attention=d_hidden_tri_attention,
        n_head_tri_attention=n_head_tri_attention,
        p_drop=0.0,
        use_triangle_attention=use_triangle_attention,
        model=triangle_model,
        d_single=d_single,
        n_head_single=n_head_single,
        single_gate_bias=single_gate_bias,
        pair_transition_n=pair_transition_n,
        single_transition_n=single_transition_n,
        parallel=parallel,
        masked_update=masked_update,
    )
    return finish(PairformerBlock(config), precision, norm_eps=norm_eps)
