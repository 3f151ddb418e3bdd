"""Host-side counts of which backend served each engine op module, and which calls it refused.

The counts live in one registry keyed weakly by module (a module that is freed takes its
counts with it) and are filled by the op classes' dispatch when a module is guarded
(:func:`foldforge_b200.engine.policy.guard`). They count Python-level calls (eager runs and
the call recorded while a CUDA graph is captured), never graph replays, and are not a
kernel trace. :func:`report_observations` returns the record FoldForge's serving report
uses (``src/foldforge/modules/engine/serving.py:36-79``: the same keys per module).
"""

from __future__ import annotations

import weakref
from collections import Counter
from typing import Any

import torch

#: module -> Counter over ("served", backend) and ("refused", reason)
_COUNTS: weakref.WeakKeyDictionary[torch.nn.Module, Counter] = weakref.WeakKeyDictionary()


def observe_call(module: torch.nn.Module, backend: str, refusal: str | None, served_by: str = "pytorch") -> None:
    """Count one call of ``module``: served by ``backend``, or refused for ``refusal`` and served by ``served_by``."""
    if torch.compiler.is_compiling():
        return  # a traced region has no per-call host observation
    counts = _COUNTS.setdefault(module, Counter())
    if refusal is None:
        counts[("served", backend)] += 1
    else:
        counts[("refused", refusal)] += 1
        counts[("served", served_by)] += 1


def reset_observations(model: torch.nn.Module) -> None:
    """Forget the counts of every module of ``model``."""
    for module in model.modules():
        _COUNTS.pop(module, None)


def _split(counts: Counter | None, kind: str) -> dict[str, int]:
    if counts is None:
        return {}
    return {key: n for (k, key), n in counts.items() if k == kind}


def report_observations(model: torch.nn.Module) -> dict[str, Any]:
    """Every guarded or observed module of ``model``: its class, selected backend and counts."""
    modules: dict[str, dict[str, Any]] = {}
    for name, module in model.named_modules():
        counts = _COUNTS.get(module)
        if counts is None and not module.__dict__.get("_ffb_guarded", False):
            continue
        modules[name or "<root>"] = {
            "class": type(module).__name__,
            "backend": getattr(module, "backend", None),
            "host_observed": counts is not None,
            "served_host_calls": _split(counts, "served"),
            "refused_host_calls": _split(counts, "refused"),
        }
    return {
        "coverage": "engine_modules_with_a_backend_guard",
        "counting": "host_calls_including_capture; excludes_compiled_regions_and_graph_replays",
        "selections_are_kernel_traces": False,
        "modules": modules,
    }
