"""The CPU oracle of the MSA-stack block reproduces the reference's own ``EvoformerBlock``.

``tests/golden/evo_*.npz`` were written by ``tests/golden/make_golden.py`` from FoldForge's
released-layout ``EvoformerBlock`` with AF3's spec (``legacy/pairformer.py:233-356``) on
weights drawn here in the engine schema (the reference's converter maps them back bitwise)
and seeded MSA / pair inputs. The oracle must match them at the reference's own fp32 parity
tolerance (``tests/models/test_engine_graph.py:27``), per op and for the whole block, on every
position; a planted mistake (the outer product's left and right swapped) must not.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle.msa as omsa
from foldforge_b200.synthetic import evoformer_state, msa_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("evo_*.npz"))
TOL = {"rtol": 1e-4, "atol": 1e-4}


def _digest(state):
    h = hashlib.sha256()
    for k in sorted(state):
        h.update(k.encode())
        h.update(state[k].contiguous().numpy().tobytes())
    return h.hexdigest()


def load(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    state = evoformer_state(torch.Generator().manual_seed(int(rec["wseed"])), scheme=str(rec["scheme"]))
    msa, z, msa_mask, tokens = msa_inputs(int(rec["n_seq"]), int(rec["n"]), int(rec["iseed"]),
                                          masked_suffix=int(rec["masked"]))
    return rec, state, msa, z, msa_mask, tokens


def sub(state, prefix):
    return {k[len(prefix) + 1:]: v for k, v in state.items() if k.startswith(prefix + ".")}


def test_there_are_msa_cases():
    assert len(CASES) >= 2


@pytest.mark.parametrize("name", CASES)
def test_seeds_reproduce_the_recorded_weights_and_inputs(name):
    rec, state, msa, z, msa_mask, _ = load(name)
    assert _digest(state) == str(rec["weights_sha256"])
    assert _digest({"msa": msa, "z": z, "msa_mask": msa_mask}) == str(rec["inputs_sha256"])


@pytest.mark.parametrize("name", CASES)
def test_ops_match_the_reference(name):
    rec, state, msa, z, msa_mask, _ = load(name)
    opm = omsa.outer_product_mean(msa, msa_mask, sub(state, "outer_product_mean"))
    torch.testing.assert_close(opm, torch.from_numpy(rec["op.outer_product_mean"]), **TOL)
    pwa = omsa.pair_weighted_averaging(msa, msa_mask, z, sub(state, "msa_attention1"))
    torch.testing.assert_close(pwa, torch.from_numpy(rec["op.msa_attention1"]), **TOL)


@pytest.mark.parametrize("name", CASES)
def test_block_matches_the_reference_everywhere(name):
    rec, state, msa, z, msa_mask, tokens = load(name)
    out_msa, out_pair = omsa.evoformer_block(msa, z, msa_mask, tokens, state)
    torch.testing.assert_close(out_msa, torch.from_numpy(rec["out_msa"]), **TOL)
    torch.testing.assert_close(out_pair, torch.from_numpy(rec["out_pair"]), **TOL)


def test_a_planted_mistake_is_caught():
    rec, state, msa, z, msa_mask, _ = load(CASES[0])
    p = sub(state, "outer_product_mean")
    p["to_left.weight"], p["to_right.weight"] = p["to_right.weight"], p["to_left.weight"]
    wrong = omsa.outer_product_mean(msa, msa_mask, p)
    with pytest.raises(AssertionError):
        torch.testing.assert_close(wrong, torch.from_numpy(rec["op.outer_product_mean"]), **TOL)
