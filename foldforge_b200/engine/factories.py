"""Factories of the engine classes, with FoldForge's choices (``src/foldforge/modules/engine/modules.py``).

Model keys, parameter precision (``master``: fp32 masters, bf16 activations; ``fp32``) and
the masks. Every factory builds on ``pytorch``; :func:`foldforge_b200.engine.policy.apply_plan`
gives the modules their backend afterwards.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch
from torch import nn

from foldforge_b200.engine.modules import (
    LayerNorm,
    MasterWeights,
    Transition,
    TriangleAttention,
    TriangleMultiplication,
)

Precision = Literal["master", "fp32"]
PRECISIONS = ("master", "fp32")


@dataclass(frozen=True)
class ModelKeys:
    """The engine selector keys of one family (``modules.py:45-58``)."""

    triangle: str | None
    token_dit: str | None = None
    atom_dit: str | None = None
    triangle_multiplication: str | None = None
    confidence: str | None = None


#: Families whose Pairformer pair stack this package builds (AF3's; the other families'
#: variants -- transposed bias, RF3 division, Chai-1 gates -- are not built here).
MODEL_KEYS: dict[str, ModelKeys] = {"alphafold3": ModelKeys("af3", "af3", "af3")}


def model_keys(family: str) -> ModelKeys:
    """The selector keys of ``family``."""
    try:
        return MODEL_KEYS[family]
    except KeyError:
        known = ", ".join(sorted(MODEL_KEYS))
        raise ValueError(f"no engine selector keys for family {family!r}; known: {known}") from None


def set_norm_eps(module: nn.Module, eps: float) -> None:
    """Set ``eps`` on every LayerNorm of ``module`` that still has the default 1e-5."""
    for sub in module.modules():
        if isinstance(sub, torch.nn.LayerNorm) and sub.eps == 1e-5:
            sub.eps = eps


def finish[M: nn.Module](module: M, precision: Precision = "master", *, norm_eps: float | None = None) -> M:
    """``master`` pins fp32 masters (``set_master_weights``), ``fp32`` is plain fp32 (``modules.py:115-129``)."""
    if precision not in PRECISIONS:
        raise ValueError(f"precision must be one of {PRECISIONS}, got {precision!r}")
    if precision == "master" and isinstance(module, MasterWeights):
        module.set_master_weights()
    else:
        module.float()
    if norm_eps is not None:
        set_norm_eps(module, norm_eps)
    return module


def transition(d_hidden: int, n: int = 4, *, precision: Precision = "master", norm_eps: float | None = None) -> Transition:
    """``Transition`` (residual included)."""
    return finish(Transition(d_hidden, n), precision, norm_eps=norm_eps)


def triangle_multiplication(d_pair: int, *, outgoing: bool, d_hidden: int | None = None, divide_by_length: bool = False,
                            precision: Precision = "master", norm_eps: float | None = None) -> nn.Module:
    """``TriangleMultiplication`` (residual included); RoseTTAFold3's length division is not built."""
    if divide_by_length:
        raise ValueError("the length-divided (RoseTTAFold3 exact) triangle multiplication is not built here")
    module = TriangleMultiplication(d_pair, d_hidden=d_hidden, outgoing=outgoing, p_drop=0.0, model=None)
    return finish(module, precision, norm_eps=norm_eps)


def triangle_attention(d_pair: int, n_head: int, *, starting: bool, model: str, d_hidden: int | None = None,
                       precision: Precision = "master", norm_eps: float | None = None) -> nn.Module:
    """``TriangleAttention(model=...)`` (residual included); ``d_hidden`` is the per-head width."""
    module = TriangleAttention(d_pair, n_head, d_hidden=d_hidden, starting=starting, p_drop=0.0, model=model)
    return finish(module, precision, norm_eps=norm_eps)


def layer_norm(d, *, eps: float = 1e-5, bias: bool = True, elementwise_affine: bool = True) -> LayerNorm:
    """The engine ``LayerNorm`` (fp32 affine under any cast)."""
    return LayerNorm(d, eps=eps, bias=bias, elementwise_affine=elementwise_affine)


def token_mask(pair_mask: torch.Tensor | None) -> torch.Tensor | None:
    """Token masks from outer-product pair masks with any leading batch axes (no host sync)."""
    if pair_mask is None:
        return None
    return (pair_mask.diagonal(dim1=-2, dim2=-1) > 0).contiguous()


def residue_mask(pair_mask: torch.Tensor | None) -> torch.Tensor | None:
    """Key mask ``[1, L]`` (bool) from an outer-product pair mask ``[L, L]``."""
    mask = token_mask(pair_mask)
    return None if mask is None else mask[None]
