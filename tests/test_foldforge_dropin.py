"""FoldForge's OWN backend policy drives the ``b200`` classes (CPU; the reference tree is needed).

The drop-in claim is that FoldForge needs one added name and no other change: its
``modules/engine/backends.py`` with ``"b200"`` appended to ``ENGINE_BACKENDS`` (line 29), and
its unmodified ``policy.py`` and ``serving.py``, applied to this package's engine classes
(which FoldForge would import in place of the absent ``miniworld_engine`` ones). This test
loads exactly those three reference files from a FoldForge checkout (``FOLDFORGE_SRC``, by
default a checkout named ``reference`` beside this repository), edits the one line in the source text,
and checks what the reference's own test of the policy checks
(``tests/kernels/test_backends.py``): the plan names, per-op pinning through ``engine.ops``,
the per-class choice, the guard's fallback with one log line, ``engine.unsupported: error``,
composite blocks set child by child, and the observations record. Without a GPU every
``b200`` call is refused by ``unsupported()`` (a CPU tensor), so the fallback path is the one
exercised; the GPU tests run the same classes on the kernels. Skipped where the reference
tree is absent (GPU boxes).
"""

from __future__ import annotations

import importlib.util
import logging
import os
import sys
import types
from pathlib import Path

import pytest
import torch
from torch import nn

from foldforge_b200.engine import modules as ours
from foldforge_b200.engine.pairformer import pairformer_block

# a FoldForge checkout: FOLDFORGE_SRC, else one named `reference` beside this repository
SRC = Path(os.environ.get("FOLDFORGE_SRC", Path(__file__).resolve().parents[2] / "reference" / "src"))
ENGINE = SRC / "foldforge" / "modules" / "engine"

pytestmark = pytest.mark.skipif(not (ENGINE / "policy.py").exists(), reason="FoldForge source tree not present")


class _ForeignOp(nn.Module):
    """Stand-in for an engine class outside the pair stack (it has only the engine's own backends)."""

    backends = ("pytorch", "cuda", "triton")


def _load(name: str, path: Path, edit=None) -> types.ModuleType:
    text = path.read_text()
    if edit is not None:
        text = edit(text)
    module = types.ModuleType(name)
    module.__file__ = str(path)
    sys.modules[name] = module
    exec(compile(text, str(path), "exec"), module.__dict__)  # noqa: S102 - the reference's own file
    return module


@pytest.fixture(scope="module")
def ff():
    """FoldForge's backends / policy / serving, bound to this package's classes."""
    saved = {k: v for k, v in sys.modules.items() if k.startswith(("foldforge.", "miniworld_engine")) or k == "foldforge"}
    engine_pkg = types.ModuleType("miniworld_engine")
    engine_mods = types.ModuleType("miniworld_engine.modules")
    for cls in (ours.TriangleMultiplication, ours.TriangleAttention, ours.TriangleAttentionAF3, ours.Transition,
                ours.AttentionPairBias, ours.LayerNorm, ours.PairformerBlock):
        setattr(engine_mods, cls.__name__, cls)
    for name in ("OuterProductMean", "MSAPairWeightedAveraging", "ConditionedTransition", "TokenDiTProtenix",
                 "AtomDiTProtenix", "AugmentNoise"):
        setattr(engine_mods, name, type(name, (_ForeignOp,), {}))
    engine_pkg.modules = engine_mods
    sys.modules.update({"miniworld_engine": engine_pkg, "miniworld_engine.modules": engine_mods})
    for pkg in ("foldforge", "foldforge.modules", "foldforge.modules.engine"):
        sys.modules[pkg] = types.ModuleType(pkg)

    def add_b200(text: str) -> str:
        line = 'ENGINE_BACKENDS = ("pytorch", "cuda", "triton", "anthropic", "cueq")'
        assert text.count(line) == 1, "the reference's ENGINE_BACKENDS line moved"
        return text.replace(line, line[:-1] + ', "b200")')

    backends = _load("foldforge.modules.engine.backends", ENGINE / "backends.py", add_b200)
    serving = _load("foldforge.modules.engine.serving", ENGINE / "serving.py")
    policy = _load("foldforge.modules.engine.policy", ENGINE / "policy.py")
    yield types.SimpleNamespace(backends=backends, policy=policy, serving=serving)
    for k in [k for k in sys.modules if k.startswith(("foldforge.", "miniworld_engine")) or k == "foldforge"]:
        del sys.modules[k]
    sys.modules.update(saved)


@pytest.fixture(autouse=True)
def _fresh(ff):
    ff.policy.forget_logged_refusals()


class _Model(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.transition = ours.Transition(128, 4)
        self.trimul = ours.TriangleMultiplication(128, 128, outgoing=True)
        self.norm = ours.LayerNorm(128)


def _x() -> torch.Tensor:
    return torch.randn(1, 6, 6, 128, generator=torch.Generator().manual_seed(0))


def test_the_added_name_is_a_backend_and_serves_the_pair_ops(ff):
    assert "b200" in ff.backends.ENGINE_BACKENDS and "b200" in ff.backends.BACKENDS
    plan = ff.backends.BackendPlan.make("b200", {"transition": "pytorch"})
    assert plan.requested("trimul") == "b200" and plan.requested("transition") == "pytorch"
    serves = ff.backends.SERVES
    for op in ("trimul", "triangle_attention", "single_attention", "transition", "layernorm"):
        assert "b200" in serves[op], (op, serves[op])
    assert ff.backends.choose_backend("b200", ours.Transition, torch.device("cpu")) == ("b200", None)
    name, why = ff.backends.choose_backend("cuda", ours.Transition, torch.device("cpu"))
    assert name == "pytorch" and "no 'cuda' backend" in why
    with pytest.raises(ValueError):
        ff.backends.BackendPlan.make("b300")


def test_resolve_names_the_ops_no_class_serves(ff, caplog):
    plan = ff.backends.BackendPlan.make("b200")
    with caplog.at_level(logging.WARNING, logger="foldforge.backend"):
        plan.resolve(torch.device("cpu"))
    assert plan.of("trimul") == "b200" and plan.of("triangle_attention") == "b200"
    assert plan.report()["fallbacks"].keys() >= {"opm", "msa_pwa"}
    assert "trimul" not in plan.report()["fallbacks"]
    with pytest.raises(ff.backends.BackendUnsupportedError):
        ff.backends.BackendPlan.make("pytorch", {"opm": "b200"}, "error").resolve(torch.device("cpu"))


def test_engine_ops_pins_one_op(ff):
    model = _Model()
    choices = ff.policy.apply_plan(model, ff.backends.BackendPlan.make("pytorch", {"trimul": "b200"}),
                                   torch.device("cpu"))
    assert (model.trimul.backend, model.transition.backend, model.norm.backend) == ("b200", "pytorch", "pytorch")
    assert choices["trimul"] == {"op": "trimul", "backend": "b200", "requested": "b200", "reason": None}


def test_a_refused_call_falls_back_to_pytorch_once_logged(ff, caplog):
    model = _Model()
    x = _x()
    expected = model.transition(x)  # pytorch backend, before any plan
    ff.policy.apply_plan(model, ff.backends.BackendPlan.make("b200"), torch.device("cpu"))
    assert model.transition.backend == "b200"
    assert model.transition.unsupported(x) == "tensor is not on a CUDA device"
    with caplog.at_level(logging.WARNING, logger="foldforge.backend"):
        first, second = model.transition(x), model.transition(x)
    torch.testing.assert_close(first, expected)
    torch.testing.assert_close(second, expected)
    assert model.transition.backend == "b200"
    assert sum("refuses a call" in r.message for r in caplog.records) == 1
    record = ff.serving.report_observations(model)["modules"]["transition"]
    assert record["served_host_calls"] == {"pytorch": 2}
    assert record["refused_host_calls"] == {"tensor is not on a CUDA device": 2}


def test_unsupported_error_raises_foldforge_error(ff):
    model = _Model()
    ff.policy.apply_plan(model, ff.backends.BackendPlan.make("b200", unsupported="error"), torch.device("cpu"))
    with pytest.raises(ff.backends.BackendUnsupportedError, match="engine.unsupported: error"):
        model.trimul(_x())


def test_pairformer_block_children_are_set_one_by_one(ff):
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, precision="fp32")
    holder = nn.ModuleList([block])
    choices = ff.policy.apply_plan(holder, ff.backends.BackendPlan.make("b200", {"single_attention": "pytorch"}),
                                   torch.device("cpu"))
    assert block.backend == "pytorch"
    assert block.tri_multi_outgoing.backend == "b200" and block.tri_atten_ending.backend == "b200"
    assert block.single_attention.backend == "pytorch"
    assert set(choices) == {f"0.{n}" for n in ("tri_multi_outgoing", "tri_multi_incoming", "tri_atten_starting",
                                               "tri_atten_ending", "transition_pair", "single_attention",
                                               "single_transition")}
    z = torch.randn(1, 5, 5, 128, generator=torch.Generator().manual_seed(1))
    s = torch.randn(1, 5, 384, generator=torch.Generator().manual_seed(2))
    mask = torch.ones(1, 5, dtype=torch.bool)
    pair, single = block(z, mask, s)  # every pair op refused on the CPU, served by pytorch
    assert pair.shape == z.shape and single.shape == s.shape
    served = {k: v["served_host_calls"] for k, v in ff.serving.report_observations(holder)["modules"].items()}
    assert all(v == {"pytorch": 1} for v in served.values()), served
