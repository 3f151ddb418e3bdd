"""Which backend serves which op: the table behind ``backend``, ``engine.ops`` and ``engine.unsupported``.

Mirrors FoldForge's policy module (``src/foldforge/modules/engine/backends.py:29-271``) for
the Pairformer pair stack, with one backend name added: ``b200`` (the sm_100a kernels of
this package). The reference engine's own names (``cuda``, ``triton``, ``anthropic``,
``cueq``) stay VALID configuration values, so an existing FoldForge config parses, but no
class here has them: asking for one is a refusal that runs ``pytorch`` with a reason, as the
reference does for a class that lacks a backend (``choose_backend``, ``:137-165``).

* ``Config.backend`` takes the backend names plus the policy alias ``miniworld`` = "the
  engine's own kernels": here ``b200`` where the class has it and an sm_100 device exists,
  else ``pytorch`` (not a refusal).
* ``engine.ops`` pins single ops (the keys of ``OP_CLASSES``) to another backend.
* ``engine.unsupported``: ``fallback`` (default) runs the ``pytorch`` backend of that module
  for a call the chosen backend refuses, with ONE log line; ``error`` raises.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import TYPE_CHECKING

if TYPE_CHECKING:
    from collections.abc import Mapping

logger = logging.getLogger("foldforge.backend")

#: Backends a class of this package can have.
ENGINE_BACKENDS = ("pytorch", "b200")
#: The reference engine's kernel backends: valid names, served by no class here.
FOREIGN_BACKENDS = ("cuda", "triton", "anthropic", "cueq")
#: Policy aliases of ``Config.backend``; ``None`` = decided per class by :func:`choose_backend`.
ALIASES: dict[str, str | None] = {"miniworld": None, "cuequivariance": "cueq"}
BACKENDS = ("miniworld", "cuequivariance", *ENGINE_BACKENDS, *FOREIGN_BACKENDS)

#: op -> the engine classes (by name, in :mod:`foldforge_b200.engine.modules`) that carry it.
#: The keys are the names ``engine.ops`` takes (``backends.py:35-70``); ops outside the
#: Pairformer pair stack have no class in this package.
OP_CLASSES: dict[str, tuple[str, ...]] = {
    "trimul": ("TriangleMultiplication",),
    "triangle_attention": ("TriangleAttention", "TriangleAttentionAF3"),
    "opm": (),
    "msa_pwa": (),
    "single_attention": ("AttentionPairBias",),
    "transition": ("Transition",),
    "layernorm": ("LayerNorm",),
    "conditioning": (),
    "dit_blocks": (),
    "atom_blocks": (),
    "sampler_ops": (),
}
OPS = tuple(OP_CLASSES)
UNSUPPORTED = ("fallback", "error")
#: The compute capability the ``b200`` kernels are built for (sm_100a).
B200_CAPABILITY = (10, 0)


class BackendUnsupportedError(RuntimeError):
    """A (backend, module) combination nothing serves, with ``engine.unsupported: error``."""


def op_classes(op: str) -> tuple[type, ...]:
    """The engine classes of ``op``."""
    from foldforge_b200.engine import modules

    return tuple(getattr(modules, name) for name in OP_CLASSES[op] if hasattr(modules, name))


def op_of(module: object) -> str | None:
    """The op an engine module instance carries, or None."""
    for op in OPS:
        classes = op_classes(op)
        if classes and isinstance(module, classes):
            return op
    return None


def serves(op: str) -> tuple[str, ...]:
    """The backends some class of ``op`` has, in the policy's names (``miniworld`` when any has ``b200``)."""
    have = {b for cls in op_classes(op) for b in cls.backends}
    named = [b for b in ENGINE_BACKENDS if b in have]
    return (*(["miniworld"] if "b200" in have else []), *named)


def __getattr__(name: str) -> object:
    """``SERVES``: op -> :func:`serves`, derived from the classes on first use."""
    if name == "SERVES":
        return {op: serves(op) for op in OPS}
    raise AttributeError(name)


def validate_ops(ops: Mapping[str, str]) -> dict[str, str]:
    """``engine.ops``: known op names, known backends."""
    unknown = sorted(set(ops) - set(OPS))
    if unknown:
        message = f"engine.ops names unknown op(s) {unknown}; known: {list(OPS)}"
        raise ValueError(message)
    bad = {op: b for op, b in ops.items() if b not in BACKENDS}
    if bad:
        message = f"engine.ops names unknown backend(s) {bad}; known: {list(BACKENDS)}"
        raise ValueError(message)
    return dict(ops)


def capability(device: object | None) -> tuple[int, int] | None:
    """The compute capability of a CUDA ``device`` (None without CUDA)."""
    import torch

    if not torch.cuda.is_available() or getattr(device, "type", "cuda") != "cuda":
        return None
    index = getattr(device, "index", None)
    return torch.cuda.get_device_capability(index)


def choose_backend(requested: str, cls: type, device: object | None = None) -> tuple[str, str | None]:
    """``(backend, reason)`` of one class: the backend it runs under ``requested`` and, when
    that is not what was asked for, why (``backends.py:137-165`` with ``b200`` in place of
    the engine's ``cuda``)."""
    name = ALIASES.get(requested, requested)
    have = tuple(cls.backends)
    cc = capability(device)
    if name is None:
        if "b200" in have and cc == B200_CAPABILITY:
            return "b200", None
        return "pytorch", None
    if name == "pytorch":
        return "pytorch", None
    if name not in have:
        return "pytorch", f"{cls.__name__} has no {name!r} backend (available: {', '.join(have)})"
    if name == "b200" and cc is None:
        return "pytorch", "the b200 backend needs a CUDA device"
    if name == "b200" and cc != B200_CAPABILITY:
        return "pytorch", f"the b200 backend needs an sm_100 device (this one is sm_{cc[0]}{cc[1]})"
    return name, None


@dataclass(frozen=True)
class Resolved:
    """One op after the checks: what was asked, what runs, and why they differ."""

    op: str
    requested: str
    backend: str
    reason: str | None = None


@dataclass(frozen=True)
class BackendPlan:
    """The backend of every op for one loaded model (``backends.py:178-271``)."""

    backend: str = "miniworld"
    ops: tuple[tuple[str, str], ...] = ()
    unsupported: str = "fallback"
    resolved: dict[str, Resolved] = field(default_factory=dict, compare=False, hash=False)

    @classmethod
    def make(cls, backend: str = "miniworld", ops: Mapping[str, str] | None = None,
             unsupported: str = "fallback") -> BackendPlan:
        """A plan; ``backend`` and ``ops`` are validated here."""
        if backend not in BACKENDS:
            message = f"Unknown backend: {backend}"
            raise ValueError(message)
        if unsupported not in UNSUPPORTED:
            message = f"engine.unsupported must be one of {UNSUPPORTED}, got {unsupported!r}"
            raise ValueError(message)
        return cls(backend, tuple(sorted(validate_ops(ops or {}).items())), unsupported)

    def requested(self, op: str) -> str:
        """The backend asked for ``op``: its ``engine.ops`` entry, else ``backend``."""
        return dict(self.ops).get(op, self.backend)

    def of(self, op: str) -> str:
        """The backend that runs ``op`` (after :meth:`resolve`)."""
        resolved = self.resolved.get(op)
        return resolved.backend if resolved is not None else self.requested(op)

    def uses(self, *backends: str) -> bool:
        """Whether any op is asked to run on one of ``backends``."""
        names = {ALIASES.get(b, b) or b for b in backends} | set(backends)
        return any(self.requested(op) in names or ALIASES.get(self.requested(op)) in names for op in OPS)

    def for_class(self, cls: type, device: object | None = None) -> tuple[str, str | None]:
        """:func:`choose_backend` for ``cls`` under this plan's request for its op."""
        op = next(op for op in OPS if op_classes(op) and issubclass(cls, op_classes(op)))
        return choose_backend(self.requested(op), cls, device)

    def resolve(self, device: object | None = None) -> BackendPlan:
        """Check every op against the classes and the machine; fill ``resolved``; apply ``unsupported``."""
        self.resolved.clear()
        for op in OPS:
            asked = self.requested(op)
            classes = op_classes(op)
            if not classes:
                continue  # no class of this package carries the op
            choices = [choose_backend(asked, cls, device) for cls in classes]
            ok = [name for name, reason in choices if reason is None]
            if ok:
                self.resolved[op] = Resolved(op, asked, ok[0])
            else:
                self.resolved[op] = Resolved(op, asked, "pytorch", choices[0][1])
        missing = [r for r in self.resolved.values() if r.reason is not None]
        if missing and self.unsupported == "error":
            lines = "; ".join(f"{r.op} on {r.requested}: {r.reason}" for r in missing)
            message = f"backend ops no engine class serves (engine.unsupported: error): {lines}"
            raise BackendUnsupportedError(message)
        if missing:
            lines = "; ".join(f"{r.op} ({r.requested}: {r.reason})" for r in missing)
            logger.warning("backend %s: running the engine pytorch backend for %s", self.backend, lines)
        return self

    def report(self) -> dict[str, object]:
        """The load report's record: the backend of every op and each refusal's reason."""
        return {
            "backend": self.backend,
            "ops": {op: r.backend for op, r in self.resolved.items()},
            "fallbacks": {op: f"{r.requested}: {r.reason}" for op, r in self.resolved.items() if r.reason is not None},
            "unsupported": self.unsupported,
        }
