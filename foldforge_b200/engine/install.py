"""Gives a loaded model's op modules their backends (``src/foldforge/modules/engine/install.py:37-64``)."""

from __future__ import annotations

from collections.abc import Collection
from typing import Any

import torch
from torch import nn

from foldforge_b200.engine.backends import BackendPlan
from foldforge_b200.engine.policy import apply_plan


def install_engine(model: nn.Module, device: str | torch.device, *, modules: bool = True, skip: Collection[str] = (),
                   plan: BackendPlan | None = None) -> nn.Module:
    """Apply ``plan`` (default: ``miniworld`` everywhere) to ``model``'s op modules and record
    the plan and per-module choices in ``model.foldforge_load_report["engine_backends"]``."""
    plan = BackendPlan.make() if plan is None else plan
    if not modules or "engine_modules" in set(skip):
        plan = BackendPlan.make("pytorch", None, plan.unsupported)
    plan.resolve(torch.device(device))
    choices = apply_plan(model, plan, torch.device(device))
    report: dict[str, Any] = getattr(model, "foldforge_load_report", {})
    report["engine_backends"] = {"plan": plan.report(), "modules": choices}
    model.foldforge_load_report = report
    return model
