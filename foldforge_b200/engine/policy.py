"""Applying a backend plan to a model, and the ``engine.unsupported`` policy for refused calls.

FoldForge's policy (``src/foldforge/modules/engine/policy.py:77-155``) guards each engine op
module: before a call it asks ``module.unsupported(*args)``; a reason runs the ``pytorch``
backend (``fallback``, one log line per distinct refusal) or raises (``error``). This
package keeps that contract and these names (:func:`apply_plan`, :func:`guard`,
:func:`refuse`, :func:`fallback_backend`, :func:`forget_logged_refusals`), but the guard is
not a wrapper around ``forward``: the op classes of :mod:`foldforge_b200.engine.modules`
dispatch every call themselves, and a guarded module's dispatch consults this module (the
policy is the module attribute ``foldforge_unsupported``). FoldForge's own guard, which
wraps ``forward`` and calls ``_forward_<backend>``, works on the same classes unchanged.

:func:`apply_plan` gives each op module the backend the plan chose for its class; composite
blocks (``PairformerBlock``, ``Pairformer``) stay ``pytorch`` themselves and their op
children are set one by one, so a refused op is refused alone.
"""

from __future__ import annotations

import logging
from typing import TYPE_CHECKING, Any

from foldforge_b200.engine.backends import BackendPlan, BackendUnsupportedError, op_of

if TYPE_CHECKING:
    from torch import nn

logger = logging.getLogger("foldforge.backend")

_COMPOSITES = frozenset(("PairformerBlock", "Pairformer"))
GUARDED_ATTR = "_ffb_guarded"


class _RefusalLog:
    """Refusals already reported, so that each (class, backend, reason) is logged once."""

    def __init__(self) -> None:
        self.seen: set[tuple[str, str, str]] = set()

    def first(self, cls: str, backend: str, reason: str) -> bool:
        key = (cls, backend, reason)
        if key in self.seen:
            return False
        self.seen.add(key)
        return True


_LOG = _RefusalLog()


def forget_logged_refusals() -> None:
    """Log every refusal again from now on (tests; a server that wants one line per request)."""
    _LOG.seen.clear()


def refuse(module: nn.Module, reason: str, served_by: str = "pytorch") -> bool:
    """Apply the module's ``engine.unsupported`` policy to a refused call: raise
    :class:`BackendUnsupportedError` under ``error``; under ``fallback`` log the refusal the
    first time it is seen and return True (the caller runs ``served_by``)."""
    cls, backend = type(module).__name__, str(module.backend)
    if getattr(module, "foldforge_unsupported", "fallback") == "error":
        raise BackendUnsupportedError(f"{cls} backend {backend!r} refuses a call (engine.unsupported: error): {reason}")
    if _LOG.first(cls, backend, reason):
        logger.warning("%s backend %s refuses a call: %s; running its %s backend for it", cls, backend, reason,
                       served_by)
    return True


def fallback_backend(module: nn.Module, backend: str, *args: Any, **kwargs: Any) -> str:
    """The backend a call refused by ``backend`` runs: the reference ``pytorch`` (the ``b200``
    kernels have no intermediate rung to fall to)."""
    del module, backend, args, kwargs
    return "pytorch"


def guard(module: nn.Module, unsupported: str = "fallback") -> nn.Module:
    """Put ``module`` under the ``unsupported`` policy (idempotent; the policy is read per call).

    The module's own dispatch then asks ``unsupported(...)`` before every call and follows
    the policy; the op classes of this package all dispatch that way."""
    if not getattr(type(module), "dispatches_policy", False):
        raise TypeError(f"{type(module).__name__} does not dispatch through the backend policy")
    module.foldforge_unsupported = unsupported
    object.__setattr__(module, GUARDED_ATTR, True)
    return module


def apply_plan(model: nn.Module, plan: BackendPlan, device: object | None = None) -> dict[str, dict[str, str | None]]:
    """Give every op module of ``model`` its backend under ``plan`` and guard it; returns
    ``{module name: {"op", "backend", "requested", "reason"}}`` (op modules are not descended
    into: their parts are parameter holders, not ops)."""
    report: dict[str, dict[str, str | None]] = {}
    stack: list[tuple[str, nn.Module]] = [("", model)]
    while stack:
        name, module = stack.pop()
        op = None if type(module).__name__ in _COMPOSITES else op_of(module)
        if op is None:
            if type(module).__name__ in _COMPOSITES and hasattr(module, "set_backend"):
                module.set_backend("pytorch")
                module.foldforge_unsupported = plan.unsupported
            children = [(f"{name}.{n}" if name else n, child) for n, child in module.named_children()]
            stack.extend(reversed(children))
            continue
        backend, reason = plan.for_class(type(module), device)
        if reason is not None and plan.unsupported == "error":
            raise BackendUnsupportedError(f"{name or '<root>'} ({type(module).__name__}): {reason}")
        module.set_backend(backend)
        guard(module, plan.unsupported)
        report[name] = {"op": op, "backend": backend, "requested": plan.requested(op), "reason": reason}
    refused = sorted((n, r) for n, r in report.items() if r["reason"] is not None)
    if refused:
        shown = "; ".join(f"{n} ({r['requested']}: {r['reason']})" for n, r in refused[:8])
        logger.warning("backend %s: %d module(s) run the engine pytorch backend: %s%s", plan.backend, len(refused),
                       shown, " ..." if len(refused) > 8 else "")
    return report
