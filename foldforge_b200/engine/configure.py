"""Precision and device of a loaded model (``src/foldforge/modules/engine/configure.py:26-99``).

``dtype`` is the ACTIVATION dtype: bf16 means precision ``master`` (fp32 parameters, run
under :func:`activation_autocast`), fp32 means precision ``fp32``.
"""

from __future__ import annotations

import contextlib
from typing import cast

import torch
from torch import nn

from foldforge_b200.engine.backends import BACKENDS
from foldforge_b200.engine.modules import MasterWeights

_ACTIVATION_PRECISION = {torch.bfloat16: "master", torch.float32: "fp32"}


def precision_of(dtype: torch.dtype) -> str:
    """The parameter precision an activation dtype runs with (``master`` for bf16, ``fp32`` for fp32)."""
    try:
        return _ACTIVATION_PRECISION[dtype]
    except KeyError:
        raise ValueError(f"activation dtype {dtype} has no parameter precision (bfloat16 -> master, float32 -> fp32)") from None


def configure_model(model: nn.Module, backend: str = "miniworld", dtype: torch.dtype = torch.bfloat16,
                    device: str | torch.device = "cuda") -> nn.Module:
    """Move ``model`` to ``device`` keeping fp32 parameters and record its precision."""
    if backend not in BACKENDS:
        raise ValueError(f"Unknown backend: {backend}")
    precision = precision_of(dtype)
    model.to(device=device)
    if precision == "master":
        for module in model.modules():
            if isinstance(module, MasterWeights):
                module.set_master_weights()
    model.foldforge_precision = precision
    model.foldforge_activation_dtype = dtype
    model.eval().requires_grad_(requires_grad=False)
    for name, param in model.named_parameters():
        if param.dtype != torch.float32:
            raise TypeError(f"{name}: {param.dtype}; parameters are fp32 (master or plain), never native low precision")
    return model


def activation_autocast(model: nn.Module) -> contextlib.AbstractContextManager[None]:
    """The autocast a ``master`` model runs under (bf16 on its device type); a no-op otherwise."""
    if getattr(model, "foldforge_precision", None) != "master":
        return contextlib.nullcontext()
    device = next(model.parameters()).device.type
    return torch.autocast(device, dtype=cast("torch.dtype", model.foldforge_activation_dtype))


def engine_activation(tensor: torch.Tensor | None) -> torch.Tensor | None:
    """``tensor`` in the dtype the ``master`` modules are called with (the autocast dtype)."""
    if tensor is None or tensor.dtype != torch.float32 or not torch.is_autocast_enabled(tensor.device.type):
        return tensor
    return tensor.to(torch.get_autocast_dtype(tensor.device.type))
