"""The engine token DiT classes (``foldforge_b200.engine.dit``) on the CPU.

The block's state-dict keys are the converter's engine schema, and the ``pytorch`` backend
through :class:`TokenDiTStack` (the reference stack's call) reproduces the reference's own
``DiffusionTransformer`` outputs committed in ``tests/golden/dit_*.npz``.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from foldforge_b200.engine.dit import TokenDiT, TokenDiTStack
from foldforge_b200.synthetic import dit_inputs, dit_schema, dit_stack_state

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("dit_*.npz"))


def _stack(blocks):
    stack = TokenDiTStack([TokenDiT() for _ in blocks])
    for blk, st in zip(stack.blocks, blocks, strict=True):
        blk.load_state_dict(st, strict=True)
    return stack.eval()


def test_keys_are_the_engine_schema():
    assert set(TokenDiT().state_dict()) == {k for k, _ in dit_schema()}
    for k, shape in dit_schema():
        assert tuple(TokenDiT().state_dict()[k].shape) == shape


@pytest.mark.parametrize("name", CASES)
def test_pytorch_backend_matches_the_reference(name):
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    blocks = dit_stack_state(int(rec["n_blocks"]), int(rec["wseed"]), str(rec["scheme"]))
    x, cond, pair, mask = dit_inputs(int(rec["samples"]), int(rec["n"]), int(rec["iseed"]),
                                     masked_suffix=int(rec["masked"]))
    stack = _stack(blocks)
    with torch.no_grad():
        out = stack(x, mask, cond, pair)
    torch.testing.assert_close(out, torch.from_numpy(rec["out"]), rtol=1e-4, atol=1e-4)
    if x.shape[0] == 1:  # the unbatched call [L, c] gives the same
        with torch.no_grad():
            out1 = stack(x[0], mask, cond, pair)
        torch.testing.assert_close(out1, out[0])


def test_b200_is_refused_off_gpu_with_a_reason():
    blk = TokenDiT()
    blk.backend = "b200"
    x = torch.zeros(1, 1, 4, 768, dtype=torch.bfloat16)
    reason = blk.unsupported(x, torch.zeros(1, 1, 4, 384, dtype=torch.bfloat16),
                             torch.zeros(1, 4, 4, 128, dtype=torch.bfloat16))
    assert reason and "CUDA" in reason
