"""The token diffusion transformer on the b200 kernels (B200 only).

The ``b200`` backend of :class:`TokenDiTStack` (bf16 activations, master weights) against the
CPU oracle (``oracle/dit.py``, pinned to the reference's ``DiffusionTransformer``) on the same
bf16-rounded inputs: the output within relative L2 1e-2 and each block's update within 3e-2
(the bf16 rounding of the activations fed to the GEMMs), on the reference fixtures and on
larger ragged / masked shapes, including every key masked (uniform attention). The per-fold
tables are reused for the same conditioning and rebuilt after an in-place change.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
import oracle.dit as odit  # noqa: E402
from foldforge_b200.engine.dit import TokenDiT, TokenDiTStack  # noqa: E402
from foldforge_b200.synthetic import dit_inputs, dit_stack_state  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("dit_*.npz"))
DEV = torch.device("cuda")


def _stack(blocks):
    stack = TokenDiTStack([TokenDiT() for _ in blocks])
    for blk, st in zip(stack.blocks, blocks, strict=True):
        blk.load_state_dict(st, strict=True)
    stack = stack.to(DEV).eval()
    for blk in stack.blocks:
        blk.set_master_weights()
        blk.set_backend("b200")
    return stack


def _check(blocks, x, cond, pair, mask):
    xb, cb, pb = x.bfloat16(), cond.bfloat16(), pair.bfloat16()
    stack = _stack(blocks)
    with torch.no_grad():
        got = stack(xb.to(DEV), mask.to(DEV) > 0, cb.to(DEV), pb.to(DEV)).float().cpu()
    want = odit.token_dit_stack(xb.float(), cb.float(), pb.float(), mask, blocks)
    assert torch.isfinite(got).all()
    assert oracle.rel_l2(got, want) < 1e-2
    assert oracle.rel_l2(got - xb.float(), want - xb.float()) < 3e-2 * len(blocks) ** 0.5
    return stack, got


@pytest.mark.parametrize("name", CASES)
def test_matches_the_oracle_on_the_reference_fixtures(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    blocks = dit_stack_state(int(rec["n_blocks"]), int(rec["wseed"]), str(rec["scheme"]))
    x, cond, pair, mask = dit_inputs(int(rec["samples"]), int(rec["n"]), int(rec["iseed"]),
                                     masked_suffix=int(rec["masked"]))
    _check(blocks, x, cond, pair, mask)


@pytest.mark.parametrize("samples,n,masked", [(5, 100, 7), (3, 257, 0), (2, 65, 64)])
def test_matches_the_oracle_at_ragged_lengths(samples, n, masked):
    blocks = dit_stack_state(1, 21, "randomise")
    x, cond, pair, mask = dit_inputs(samples, n, 22, masked_suffix=masked)
    _check(blocks, x, cond, pair, mask)


def test_every_key_masked_averages_uniformly():
    blocks = dit_stack_state(1, 23, "randomise")
    x, cond, pair, mask = dit_inputs(2, 20, 24, masked_suffix=20)
    _check(blocks, x, cond, pair, mask)


def test_tables_are_kept_per_conditioning():
    blocks = dit_stack_state(1, 25, "randomise")
    x, cond, pair, mask = dit_inputs(2, 40, 26)
    stack = _stack(blocks)
    xb, cb, pb, m = x.bfloat16().to(DEV), cond.bfloat16().to(DEV), pair.bfloat16().to(DEV), mask.to(DEV) > 0
    with torch.no_grad():
        first = stack(xb, m, cb, pb)
        tables = stack.blocks[0]._tables[1]
        again = stack(xb, m, cb, pb)
        assert stack.blocks[0]._tables[1] is tables
        assert torch.equal(first, again)
        pb.mul_(0.5)  # an in-place change of the pair: the tables are rebuilt
        changed = stack(xb, m, cb, pb)
        assert stack.blocks[0]._tables[1] is not tables
    want = odit.token_dit_stack(xb.float().cpu(), cb.float().cpu(), pb.float().cpu(), mask, blocks)
    assert oracle.rel_l2(changed.float().cpu(), want) < 1e-2
