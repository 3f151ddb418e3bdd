"""Parity at the benchmark configurations (B200 only; minutes of CPU oracle time).

* The 48-block trunk of benchmark configuration 2 exactly as ``bench.py`` times it: N = 512,
  the last 26 tokens padded, ``trunk_state(48, seed=0, scheme="baseline")``, z and s from
  ``inputs(512, seed=0)``, master precision, ``masked_update="zero"``. The CPU oracle (fp32,
  all host threads) is stepped block by block beside it:
  - teacher-forced: block i of the b200 trunk gets the oracle's state before block i
    (rounded to bf16, as the bf16 activation stream carries it); its output must be within
    relative L2 1e-2 of the oracle's (the reference's own GPU test allows relative RMS 3e-2
    on the outputs, ``tests/kernels/test_backends_cuda.py:58-59``), and its update within
    3e-2 of the oracle's update beyond the floor that the bf16 rounding of the output alone
    sets (``hypot(3e-2, floor)``; the floor is large where the update is small next to the
    state, e.g. the single track's first blocks);
  - free-running: the b200 trunk's output after 48 blocks against the fp32 oracle's. Master
    precision stores the pair and the single in bf16 between ops (240 roundings of the pair
    per trunk), and that storage alone moves a trajectory away from the fp32 one: the oracle
    itself, run with bf16 storage between ops (exact fp32 arithmetic otherwise, i.e. an
    ideal master-mode implementation), drifts ~2.8e-2 from its fp32 run over 48 blocks. The
    bound is therefore the larger of 1e-2 (the north-star master-mode bar) and 1.25 times
    that storage floor, measured here on the same inputs; padded pairs and tokens must be
    exactly the input (``masked_update="zero"``).
* One block of the length ladder's shape class (configuration 3): N = 1024 with a 5% padded
  suffix, against the oracle.

Real positions only: in "zero" mode the padded positions keep their input, while the oracle
(the reference equations) updates them; real positions never read padded values (their keys
are masked), so both trajectories agree there. Set ``FFB_PARITY_LOG`` to a file path to get
the per-block figures as JSON.
"""

from __future__ import annotations

import json
import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
import foldforge_b200  # noqa: E402
from foldforge_b200 import _lib  # noqa: E402
from foldforge_b200.synthetic import block_state, inputs, trunk_state  # noqa: E402

UPDATE_TOL = 3e-2
OUTPUT_TOL = 1e-2


@pytest.fixture(autouse=True)
def _threads():
    old = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    yield
    torch.set_num_threads(old)


def _log(name: str, record: dict) -> None:
    path = os.environ.get("FFB_PARITY_LOG")
    if not path:
        return
    data = json.loads(open(path).read()) if os.path.exists(path) else {}
    data[name] = record
    with open(path, "w") as f:
        json.dump(data, f, indent=1)


def test_benchmark_trunk_matches_the_oracle_block_by_block():
    n, masked, nb = 512, 26, 48
    states = trunk_state(nb, seed=0, scheme="baseline")
    dev = torch.device("cuda")
    trunk = foldforge_b200.load(states, backend="b200", unsupported="error", dtype=torch.bfloat16, device=dev)
    z, s, tokens = inputs(n, 0, masked_suffix=masked)
    mask = (tokens > 0)[None].to(dev)
    pm = (tokens[:, None] * tokens[None, :]) > 0
    tk = tokens > 0
    z0, s0 = z.bfloat16(), s.bfloat16()
    zg, sg = z0[None].to(dev), s0[None].to(dev)  # free-running b200 state
    zo, so = z0.float(), s0.float()              # oracle state (fp32)
    zb, sb = z0.float(), s0.float()              # oracle with bf16 storage between ops (the floor)
    per_block = []
    for i, (st, block) in enumerate(zip(states, trunk.blocks)):
        with torch.no_grad():
            zi, si = zo.bfloat16(), so.bfloat16()  # teacher-forced input
            zt, stt = block(zi[None].to(dev), mask, si[None].to(dev))
            zg, sg = block(zg, mask, sg)
            zn, sn = oracle.pairformer_block(zo, so, tokens, st)
            zb, sb = oracle.pairformer_block(zb, sb, tokens, st, storage=torch.bfloat16)
        zt, stt = zt[0].float().cpu(), stt[0].float().cpu()
        rec = {"block": i}
        for name, got, x_in, want, x_ref, where in (("pair", zt, zi.float(), zn, zo, pm),
                                                     ("single", stt, si.float(), sn, so, tk)):
            rec[f"{name}_output"] = oracle.rel_l2(got, want, where)
            rec[f"{name}_update"] = oracle.rel_l2(got - x_in, want - x_ref, where)
            # what a kernel exact up to the bf16 rounding of its output would show
            rec[f"{name}_update_floor"] = oracle.rel_l2(want.bfloat16().float() - x_in, want - x_ref, where)
        per_block.append(rec)
        _log("trunk_n512_48", {"blocks": per_block})
        zo, so = zn, sn
        for name in ("pair", "single"):
            assert rec[f"{name}_output"] <= OUTPUT_TOL, rec
            assert rec[f"{name}_update"] <= math.hypot(UPDATE_TOL, rec[f"{name}_update_floor"]), rec
    assert _lib.device_error() == 0
    zf, sf = zg[0].float().cpu(), sg[0].float().cpu()
    final = {"pair": oracle.rel_l2(zf, zo, pm), "single": oracle.rel_l2(sf, so, tk),
             "pair_storage_floor": oracle.rel_l2(zb, zo, pm), "single_storage_floor": oracle.rel_l2(sb, so, tk)}
    _log("trunk_n512_48", {"final": final, "blocks": per_block})
    assert final["pair"] <= max(OUTPUT_TOL, 1.25 * final["pair_storage_floor"]), final
    assert final["single"] <= max(OUTPUT_TOL, 1.25 * final["single_storage_floor"]), final
    assert torch.equal(zg[0].cpu()[~pm], z0[~pm])
    assert torch.equal(sg[0].cpu()[~tk], s0[~tk])


def test_ladder_shape_block_at_n1024_matches_the_oracle():
    n = 1024
    masked = math.ceil(0.05 * n)
    state = block_state(torch.Generator().manual_seed(0), scheme="baseline")
    dev = torch.device("cuda")
    trunk = foldforge_b200.load([state], backend="b200", unsupported="error", dtype=torch.bfloat16, device=dev)
    z, s, tokens = inputs(n, 0, masked_suffix=masked)
    z0, s0 = z.bfloat16(), s.bfloat16()
    del z
    with torch.no_grad():
        zg, sg = trunk(z0[None].to(dev), (tokens > 0)[None].to(dev), s0[None].to(dev))
    assert _lib.device_error() == 0
    zg, sg = zg[0].float().cpu(), sg[0].float().cpu()
    zo, so = oracle.pairformer_block(z0.float(), s0.float(), tokens, state)
    pm = (tokens[:, None] * tokens[None, :]) > 0
    tk = tokens > 0
    rec = {}
    for name, got, x_in, want, where in (("pair", zg, z0.float(), zo, pm), ("single", sg, s0.float(), so, tk)):
        rec[f"{name}_output"] = oracle.rel_l2(got, want, where)
        rec[f"{name}_update"] = oracle.rel_l2(got - x_in, want - x_in, where)
        rec[f"{name}_update_floor"] = oracle.rel_l2(want.bfloat16().float() - x_in, want - x_in, where)
    _log("block_n1024", rec)
    for name in ("pair", "single"):
        assert rec[f"{name}_output"] <= OUTPUT_TOL, rec
        assert rec[f"{name}_update"] <= math.hypot(UPDATE_TOL, rec[f"{name}_update_floor"]), rec
    assert torch.equal(zg[~pm], z0.float()[~pm])
