"""Backend names, the op table and the per-op backend plan of the Pairformer pair stack.

FoldForge chooses a backend per engine op class (``src/foldforge/modules/engine/backends.py:29-271``
is its policy table); this package adds one name to it, ``b200`` (the sm_100a kernels). What
is kept from FoldForge is the interface: the names below (``ENGINE_BACKENDS``, ``BACKENDS``,
``OP_CLASSES``, ``BackendPlan.make / resolve / report`` ...), the configuration values they
accept and the record :meth:`BackendPlan.report` writes into a load report.

Rules (the semantics FoldForge documents for its own names, with ``b200`` where the engine
has ``cuda``):

* ``miniworld`` means "the engine's own kernels wherever this machine runs them": ``b200`` for
  a class that has it on an sm_100 device, else ``pytorch`` (not a refusal: nothing in
  particular was asked for). ``cuequivariance`` is another spelling of ``cueq``.
* A NAMED backend is a refusal when the class lacks it (``cuda`` / ``triton`` / ``anthropic``
  / ``cueq`` are valid names that no class here has) or, for ``b200``, when there is no
  sm_100 device; the op then runs ``pytorch`` and the reason is recorded.
* ``engine.ops`` pins single ops to another name; ``engine.unsupported`` is ``fallback``
  (run ``pytorch``, log once) or ``error`` (raise :class:`BackendUnsupportedError`).
"""

from __future__ import annotations

import logging
from typing import TYPE_CHECKING

if TYPE_CHECKING:
    from collections.abc import Mapping

logger = logging.getLogger("foldforge.backend")

#: Backends a class of this package can have.
ENGINE_BACKENDS = ("pytorch", "b200")
#: The reference engine's kernel backends: valid configuration values that no class here has.
FOREIGN_BACKENDS = ("cuda", "triton", "anthropic", "cueq")
#: Policy aliases: ``None`` = decided per class (the engine's own kernels where they run).
ALIASES: dict[str, str | None] = {"miniworld": None, "cuequivariance": "cueq"}
BACKENDS = ("miniworld", "cuequivariance", *ENGINE_BACKENDS, *FOREIGN_BACKENDS)

#: op (the names ``engine.ops`` takes) -> the engine classes that carry it, by class name in
#: :mod:`foldforge_b200.engine.modules`. Ops outside the pair stack keep their key and have
#: no class here.
OP_CLASSES: dict[str, tuple[str, ...]] = {
    "trimul": ("TriangleMultiplication",),
    "triangle_attention": ("TriangleAttention", "TriangleAttentionAF3"),
    "opm": ("OuterProductMean",),
    "msa_pwa": ("MSAPairWeightedAveraging",),
    "single_attention": ("AttentionPairBias",),
    "transition": ("Transition",),
    "layernorm": ("LayerNorm",),
    "conditioning": (),
    "dit_blocks": ("TokenDiT",),
    "atom_blocks": (),
    "sampler_ops": (),
}
OPS = tuple(OP_CLASSES)
UNSUPPORTED = ("fallback", "error")
#: The compute capability the ``b200`` kernels are built for (sm_100a).
B200_CAPABILITY = (10, 0)

#: class name -> op, the inverse of :data:`OP_CLASSES`
_OP_OF_CLASS = {name: op for op, names in OP_CLASSES.items() for name in names}


class BackendUnsupportedError(RuntimeError):
    """A (backend, module) combination nothing serves, with ``engine.unsupported: error``."""


#: modules of this package that define op classes
CLASS_MODULES = ("foldforge_b200.engine.modules", "foldforge_b200.engine.dit")


def op_classes(op: str) -> tuple[type, ...]:
    """The classes of this package that carry ``op`` (an op without any gives ``()``)."""
    import importlib

    found = []
    for name in OP_CLASSES[op]:
        for mod in CLASS_MODULES:
            cls = getattr(importlib.import_module(mod), name, None)
            if cls is not None:
                found.append(cls)
                break
    return tuple(found)


def op_of(module: object) -> str | None:
    """The op an engine module carries: the first class on its MRO that the table names."""
    for cls in type(module).__mro__:
        op = _OP_OF_CLASS.get(cls.__name__)
        if op is not None and cls.__module__ in CLASS_MODULES:
            return op
    return None


def serves(op: str) -> tuple[str, ...]:
    """Backends some class of ``op`` has, as policy names (``miniworld`` first when ``b200`` is among them)."""
    have: set[str] = set()
    for cls in op_classes(op):
        have.update(cls.backends)
    out = [name for name in ENGINE_BACKENDS if name in have]
    return ("miniworld", *out) if "b200" in have else tuple(out)


def __getattr__(name: str) -> object:
    """``SERVES`` (op -> :func:`serves`) is computed from the classes when first asked for."""
    if name != "SERVES":
        raise AttributeError(name)
    return {op: serves(op) for op in OPS}


def validate_ops(ops: Mapping[str, str]) -> dict[str, str]:
    """Check an ``engine.ops`` mapping: every key an op of :data:`OPS`, every value a backend name."""
    bad_ops = sorted(k for k in ops if k not in OP_CLASSES)
    if bad_ops:
        raise ValueError(f"engine.ops names unknown op(s) {bad_ops}; known: {list(OPS)}")
    bad_names = {k: v for k, v in ops.items() if v not in BACKENDS}
    if bad_names:
        raise ValueError(f"engine.ops names unknown backend(s) {bad_names}; known: {list(BACKENDS)}")
    return dict(ops)


def capability(device: object | None) -> tuple[int, int] | None:
    """``(major, minor)`` of a CUDA ``device`` (the current one for ``None``); ``None`` without CUDA."""
    import torch

    if getattr(device, "type", "cuda") != "cuda" or not torch.cuda.is_available():
        return None
    return torch.cuda.get_device_capability(getattr(device, "index", None))


def _refusal(name: str, cls: type, cc: tuple[int, int] | None) -> str | None:
    """Why class ``cls`` cannot run the named backend ``name`` here (``None``: it can)."""
    if name == "pytorch":
        return None
    if name not in cls.backends:
        return f"{cls.__name__} has no {name!r} backend (available: {', '.join(cls.backends)})"
    if name == "b200" and cc is None:
        return "the b200 backend needs a CUDA device"
    if name == "b200" and cc != B200_CAPABILITY:
        return f"the b200 backend needs an sm_100 device (this one is sm_{cc[0]}{cc[1]})"
    return None


def choose_backend(requested: str, cls: type, device: object | None = None) -> tuple[str, str | None]:
    """``(backend, reason)``: what class ``cls`` runs when ``requested`` is asked for on ``device``,
    and why that differs from the request (``None`` when it does not)."""
    name = ALIASES.get(requested, requested)
    cc = capability(device)
    if name is None:
        return ("b200" if "b200" in cls.backends and cc == B200_CAPABILITY else "pytorch"), None
    reason = _refusal(name, cls, cc)
    return ("pytorch", reason) if reason else (name, None)


class Resolved:
    """One op after :meth:`BackendPlan.resolve`: what was asked, what runs, and why they differ."""

    __slots__ = ("op", "requested", "backend", "reason")

    def __init__(self, op: str, requested: str, backend: str, reason: str | None = None) -> None:
        self.op, self.requested, self.backend, self.reason = op, requested, backend, reason

    def __repr__(self) -> str:
        return f"Resolved({self.op!r}: {self.requested!r} -> {self.backend!r}, reason={self.reason!r})"


class BackendPlan:
    """The backend of every op of one loaded model: a default name, per-op pins and the
    ``engine.unsupported`` policy. Build it with :meth:`make` (which validates), check it
    against the classes and the machine with :meth:`resolve`."""

    def __init__(self, backend: str = "miniworld", ops: tuple[tuple[str, str], ...] = (),
                 unsupported: str = "fallback") -> None:
        self.backend = backend
        self.ops = tuple(ops)
        self.unsupported = unsupported
        self._pins = dict(self.ops)
        self.resolved: dict[str, Resolved] = {}

    def __eq__(self, other: object) -> bool:
        return isinstance(other, BackendPlan) and (self.backend, self.ops, self.unsupported) == (
            other.backend, other.ops, other.unsupported)

    def __hash__(self) -> int:
        return hash((self.backend, self.ops, self.unsupported))

    @classmethod
    def make(cls, backend: str = "miniworld", ops: Mapping[str, str] | None = None,
             unsupported: str = "fallback") -> BackendPlan:
        """A validated plan (unknown backend, op or policy names raise ``ValueError``)."""
        if backend not in BACKENDS:
            raise ValueError(f"Unknown backend: {backend}")
        if unsupported not in UNSUPPORTED:
            raise ValueError(f"engine.unsupported must be one of {UNSUPPORTED}, got {unsupported!r}")
        pins = validate_ops(ops or {})
        return cls(backend, tuple(sorted(pins.items())), unsupported)

    def requested(self, op: str) -> str:
        """The name asked for ``op``: its pin, else the plan's backend."""
        return self._pins.get(op, self.backend)

    def of(self, op: str) -> str:
        """The backend that runs ``op``: resolved when :meth:`resolve` has run, else as requested."""
        entry = self.resolved.get(op)
        return self.requested(op) if entry is None else entry.backend

    def uses(self, *backends: str) -> bool:
        """Whether some op is asked to run one of ``backends`` (policy or engine names)."""
        wanted = set(backends) | {ALIASES.get(b) or b for b in backends}
        for op in OPS:
            asked = self.requested(op)
            if asked in wanted or ALIASES.get(asked) in wanted:
                return True
        return False

    def for_class(self, cls: type, device: object | None = None) -> tuple[str, str | None]:
        """:func:`choose_backend` for ``cls`` under the request for its op."""
        for klass in cls.__mro__:
            op = _OP_OF_CLASS.get(klass.__name__)
            if op is not None:
                return choose_backend(self.requested(op), cls, device)
        raise KeyError(f"{cls.__name__} carries no op of the table")

    def resolve(self, device: object | None = None) -> BackendPlan:
        """Decide every op against its classes on ``device``: an op runs the first backend one
        of its classes accepts; when none accepts, ``pytorch`` with the first class's reason.
        Ops without a class here are left out. Refused ops raise under ``error`` and are
        named in ONE warning under ``fallback``."""
        self.resolved = {}
        for op in OPS:
            classes = op_classes(op)
            if not classes:
                continue
            asked = self.requested(op)
            decisions = [choose_backend(asked, cls, device) for cls in classes]
            accepted = next((name for name, reason in decisions if reason is None), None)
            if accepted is not None:
                self.resolved[op] = Resolved(op, asked, accepted)
            else:
                self.resolved[op] = Resolved(op, asked, "pytorch", decisions[0][1])
        refused = [r for r in self.resolved.values() if r.reason is not None]
        if refused and self.unsupported == "error":
            detail = "; ".join(f"{r.op} on {r.requested}: {r.reason}" for r in refused)
            raise BackendUnsupportedError(f"backend ops no engine class serves (engine.unsupported: error): {detail}")
        if refused:
            detail = "; ".join(f"{r.op} ({r.requested}: {r.reason})" for r in refused)
            logger.warning("backend %s: running the engine pytorch backend for %s", self.backend, detail)
        return self

    def report(self) -> dict[str, object]:
        """The load report's record: ``backend``, ``ops`` (op -> backend), ``fallbacks``
        (op -> "requested: reason") and ``unsupported``."""
        return {
            "backend": self.backend,
            "ops": {op: r.backend for op, r in self.resolved.items()},
            "fallbacks": {op: f"{r.requested}: {r.reason}" for op, r in self.resolved.items() if r.reason},
            "unsupported": self.unsupported,
        }
