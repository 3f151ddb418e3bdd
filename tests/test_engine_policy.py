"""The backend policy on top of the classes' ``backends`` tuples (mirrors the reference's
``tests/kernels/test_backends.py``): names, the per-class choice, plan resolution, the guard
that implements ``engine.unsupported`` and the observations it records. No GPU needed: the
device capability is faked, and a CPU tensor is outside the ``b200`` backend's range."""

from __future__ import annotations

import logging

import pytest
import torch
from torch import nn

from foldforge_b200.engine import backends, factories, modules, policy
from foldforge_b200.engine.install import install_engine
from foldforge_b200.engine.modules import AttentionPairBias, BackendUnsupported, LayerNorm, Transition, TriangleMultiplication
from foldforge_b200.engine.pairformer import pairformer_block
from foldforge_b200.engine.serving import report_observations

B200 = (10, 0)


@pytest.fixture(autouse=True)
def _fresh_log_state():
    policy.forget_logged_refusals()


def test_names_and_aliases():
    assert set(backends.ENGINE_BACKENDS) == {"pytorch", "b200"}
    assert "b200" in backends.BACKENDS and "miniworld" in backends.BACKENDS
    for name in backends.BACKENDS:
        assert backends.BackendPlan.make(name).backend == name
    with pytest.raises(ValueError, match="Unknown backend"):
        backends.BackendPlan.make("magma")
    with pytest.raises(ValueError, match="unknown op"):
        backends.validate_ops({"nope": "pytorch"})
    with pytest.raises(ValueError, match="unknown backend"):
        backends.validate_ops({"trimul": "nope"})


def test_serves_is_derived_from_the_classes():
    table = backends.SERVES
    assert set(table) == set(backends.OPS)
    for op in ("trimul", "triangle_attention", "single_attention", "transition", "layernorm"):
        assert table[op] == ("miniworld", "pytorch", "b200")
    assert table["opm"] == ("miniworld", "pytorch", "b200")
    assert table["dit_blocks"] == ("miniworld", "pytorch", "b200")  # TokenDiT (engine/dit.py)


def test_choose_backend(monkeypatch):
    monkeypatch.setattr(backends, "capability", lambda _d: None)
    assert backends.choose_backend("miniworld", Transition) == ("pytorch", None)
    assert backends.choose_backend("pytorch", Transition) == ("pytorch", None)
    name, why = backends.choose_backend("b200", Transition)
    assert name == "pytorch" and "CUDA" in why
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    assert backends.choose_backend("miniworld", Transition) == ("b200", None)
    assert backends.choose_backend("b200", TriangleMultiplication) == ("b200", None)
    name, why = backends.choose_backend("cuda", Transition)
    assert name == "pytorch" and "no 'cuda' backend" in why
    monkeypatch.setattr(backends, "capability", lambda _d: (9, 0))
    assert backends.choose_backend("miniworld", Transition) == ("pytorch", None)
    name, why = backends.choose_backend("b200", Transition)
    assert name == "pytorch" and "sm_100" in why


def test_plan_resolve_reports_refused_ops(monkeypatch, caplog):
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    plan = backends.BackendPlan.make("pytorch", {"transition": "b200", "trimul": "cueq"})
    with caplog.at_level(logging.WARNING, logger="foldforge.backend"):
        plan.resolve()
    assert plan.of("transition") == "b200"
    assert plan.resolved["trimul"].reason is not None
    assert plan.report()["fallbacks"].keys() == {"trimul"}
    assert sum("trimul" in r.message for r in caplog.records) == 1
    with pytest.raises(backends.BackendUnsupportedError):
        backends.BackendPlan.make("pytorch", {"trimul": "cueq"}, "error").resolve()


class _Model(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.transition = factories.transition(128, 4, precision="fp32")
        self.trimul = factories.triangle_multiplication(128, outgoing=True, precision="fp32")
        self.norm = factories.layer_norm(128)


def _x() -> torch.Tensor:
    torch.manual_seed(0)
    return torch.randn(1, 6, 6, 128)


def test_apply_plan_sets_the_backend_per_module_and_guards(monkeypatch):
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    model = _Model()
    choices = policy.apply_plan(model, backends.BackendPlan.make("miniworld", {"trimul": "pytorch"}))
    assert model.transition.backend == "b200"
    assert model.norm.backend == "b200"
    assert model.trimul.backend == "pytorch"
    assert choices["transition"]["backend"] == "b200"
    assert choices["trimul"]["op"] == "trimul"


def test_unsupported_call_falls_back_once_and_logs_once(monkeypatch, caplog):
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    model = _Model()
    expected = Transition.forward(model.transition, _x())  # pytorch backend of the same weights
    unguarded = factories.transition(128, 4, precision="fp32")
    unguarded.set_backend("b200")
    with pytest.raises(BackendUnsupported):  # a direct call outside the range, no policy
        unguarded(_x())
    policy.apply_plan(model, backends.BackendPlan.make("b200"))
    assert model.transition.backend == "b200"
    assert model.transition.unsupported(_x()) is not None  # a CPU tensor is outside the b200 range
    with caplog.at_level(logging.WARNING, logger="foldforge.backend"):
        first = model.transition(_x())
        second = model.transition(_x())
    torch.testing.assert_close(first, expected)
    torch.testing.assert_close(second, expected)
    assert model.transition.backend == "b200"  # restored after the call
    assert sum("refuses a call" in r.message for r in caplog.records) == 1
    stats = report_observations(model)["modules"]["transition"]
    assert stats["served_host_calls"] == {"pytorch": 2}
    assert len(stats["refused_host_calls"]) == 1


def test_unsupported_error_policy_raises(monkeypatch):
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    model = _Model()
    policy.apply_plan(model, backends.BackendPlan.make("b200", unsupported="error"))
    with pytest.raises(backends.BackendUnsupportedError, match=r"engine.unsupported: error"):
        model.transition(_x())


def test_composite_children_are_set_one_by_one(monkeypatch):
    monkeypatch.setattr(backends, "capability", lambda _d: B200)
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, precision="fp32")
    holder = nn.ModuleList([block])
    policy.apply_plan(holder, backends.BackendPlan.make("miniworld", {"single_attention": "pytorch"}))
    assert block.backend == "pytorch"
    assert block.tri_multi_outgoing.backend == "b200"
    assert block.tri_atten_ending.backend == "b200"
    assert block.transition_pair.backend == "b200"
    assert block.single_attention.backend == "pytorch"


def test_install_engine_without_cuda_modules_runs_pytorch():
    model = _Model()
    install_engine(model, "cpu", modules=False)
    assert {m.backend for m in (model.transition, model.trimul, model.norm)} == {"pytorch"}
    report = model.foldforge_load_report["engine_backends"]
    assert report["plan"]["backend"] == "pytorch"
    assert set(report["modules"]) == {"transition", "trimul", "norm"}


def test_b200_takes_any_width_and_refuses_what_no_kernel_serves(monkeypatch):
    """Widths the tcgen05 kernels are not built for run the fp32 SIMT path, so b200 takes them;
    it refuses head widths above 64 (the SIMT attention's bound) and tensors off the GPU."""
    monkeypatch.setattr(modules, "_cuda_reason", lambda *ts: None)
    monkeypatch.setattr(modules, "_library_reason", lambda: None)
    module = factories.transition(64, 4, precision="fp32")
    module.set_backend("b200")
    assert module.unsupported(torch.randn(1, 4, 4, 64)) is None
    assert not module._tensor_cores(torch.randn(1, 4, 4, 64))
    assert module.unsupported(torch.randn(1, 4, 4, 64, dtype=torch.float16)) is not None
    apb = AttentionPairBias(384, 128, 4)  # head width 96
    apb.set_backend("b200")
    assert "head widths up to 64" in apb.unsupported(torch.randn(1, 4, 384), torch.randn(1, 4, 4, 128))
    tri = TriangleMultiplication(64, 32)
    tri.set_backend("b200")
    assert tri.unsupported(torch.randn(1, 4, 4, 64)) is None and not tri._tensor_cores(torch.randn(1, 4, 4, 64))
    with pytest.raises(BackendUnsupported):
        LayerNorm(8).set_backend("cuda")


def test_b200_refuses_cpu_tensors():
    module = factories.transition(64, 4, precision="fp32")
    module.set_backend("b200")
    assert module.unsupported(torch.randn(1, 4, 4, 64)) == "tensor is not on a CUDA device"


def test_dead_modules_return_their_residual_input():
    """``modules/dense/dead.py``: a flagged residual op returns its input unchanged when it
    runs without grad outside training; the block skips exactly that op."""
    block = pairformer_block(d_pair=128, triangle_model="af3", d_single=384, precision="fp32").eval()
    g = torch.Generator().manual_seed(3)
    z, s = torch.randn(1, 6, 6, 128, generator=g), torch.randn(1, 6, 384, generator=g)
    mask = torch.ones(1, 6, dtype=torch.bool)
    with torch.no_grad():
        live = block.tri_atten_starting(z, mask)
        block.tri_atten_starting.dead = True
        assert torch.equal(block.tri_atten_starting(z, mask), z)
        # the block with the op skipped: every other op still runs
        want = block.tri_multi_incoming(block.tri_multi_outgoing(z, mask), mask)
        want = block.transition_pair(block.tri_atten_ending(want, mask), mask)
        got_pair, _ = block(z, mask, s)
        torch.testing.assert_close(got_pair, want)
    assert not torch.equal(live, z)
    with torch.enable_grad():  # with grad the flag is ignored
        torch.testing.assert_close(block.tri_atten_starting(z, mask), live)
    block.train()
    with torch.no_grad():  # and in training
        torch.testing.assert_close(block.tri_atten_starting(z, mask), live)
    assert not hasattr(LayerNorm, "dead")  # a LayerNorm is not a residual module
