"""The CPU oracle of the token diffusion transformer reproduces the reference's own stack.

``tests/golden/dit_*.npz`` were written by ``tests/golden/make_golden.py`` from FoldForge's
released-layout ``DiffusionTransformer`` with AF3's spec (``legacy/transformer.py:136-294``),
on weights drawn here in the engine schema (the reference's converter maps them back bitwise)
and seeded inputs. The oracle must match the first block's attention and transition and the
whole stack at the reference's fp32 parity tolerance; a planted mistake must not.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle.dit as odit
from foldforge_b200.synthetic import dit_inputs, dit_stack_state

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("dit_*.npz"))
TOL = {"rtol": 1e-4, "atol": 1e-4}


def _digest(state):
    h = hashlib.sha256()
    for k in sorted(state):
        h.update(k.encode())
        h.update(state[k].contiguous().numpy().tobytes())
    return h.hexdigest()


def load(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    blocks = dit_stack_state(int(rec["n_blocks"]), int(rec["wseed"]), str(rec["scheme"]))
    x, cond, pair, mask = dit_inputs(int(rec["samples"]), int(rec["n"]), int(rec["iseed"]),
                                     masked_suffix=int(rec["masked"]))
    return rec, blocks, x, cond, pair, mask


def sub(state, prefix):
    return {k[len(prefix) + 1:]: v for k, v in state.items() if k.startswith(prefix + ".")}


def test_there_are_dit_cases():
    assert len(CASES) >= 2


@pytest.mark.parametrize("name", CASES)
def test_seeds_reproduce_the_recorded_weights_and_inputs(name):
    rec, blocks, x, cond, pair, mask = load(name)
    assert _digest({f"{i}.{k}": v for i, b in enumerate(blocks) for k, v in b.items()}) == str(rec["weights_sha256"])
    assert _digest({"x": x, "cond": cond, "pair": pair, "mask": mask}) == str(rec["inputs_sha256"])


@pytest.mark.parametrize("name", CASES)
def test_first_block_ops_match_the_reference(name):
    rec, blocks, x, cond, pair, mask = load(name)
    att_p = sub(blocks[0], "attention")
    att = odit.attention(x, cond, odit.pair_logits(pair, att_p), mask, att_p)
    torch.testing.assert_close(att, torch.from_numpy(rec["op.attention0"]), **TOL)
    tr = odit.transition(x + att, cond, sub(blocks[0], "transition"))
    torch.testing.assert_close(tr, torch.from_numpy(rec["op.transition0"]), **TOL)


@pytest.mark.parametrize("name", CASES)
def test_stack_matches_the_reference(name):
    rec, blocks, x, cond, pair, mask = load(name)
    out = odit.token_dit_stack(x, cond, pair, mask, blocks)
    torch.testing.assert_close(out, torch.from_numpy(rec["out"]), **TOL)


def test_a_planted_mistake_is_caught():
    rec, blocks, x, cond, pair, mask = load(CASES[0])
    p = dict(blocks[0])
    p["transition.expand_a.weight"], p["transition.expand_b.weight"] = p["transition.expand_b.weight"], p["transition.expand_a.weight"]
    wrong = odit.token_dit_stack(x, cond, pair, mask, [p] + blocks[1:])
    with pytest.raises(AssertionError):
        torch.testing.assert_close(wrong, torch.from_numpy(rec["out"]), **TOL)
