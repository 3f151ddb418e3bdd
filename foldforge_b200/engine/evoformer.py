"""AF3's MSA-stack block from engine parts (``src/foldforge/modules/engine/graph.py:237-309``).

The engine has no MSA block; FoldForge's graph composes one from engine ops, and this class
does the same from this package's ops so that the ``b200`` backend serves it: the outer
product mean (its raw update added here), MSA pair-weighted averaging and the MSA transition
(each owning its residual), then the pair track (two triangle multiplications, two triangle
attentions, the transition). Child names and state-dict keys are the converter's
(``legacy/released.py:722-749``). AF3's order (outer product mean first) only: the Boltz order
and Chai-1's parallel stages are not built here.
"""

from __future__ import annotations

import torch
from torch import nn

from foldforge_b200.engine import factories
from foldforge_b200.engine.modules import MSAPairWeightedAveraging, OuterProductMean, _PairOp

#: AF3's pair-count offset of the outer product mean's divisor (``legacy/primitives.py:68``)
OPM_COUNT_OFFSET = 1e-3


class EvoformerBlock(nn.Module):
    """One AF3 MSA-stack block. ``forward(msa [M, L, c_m], pair [L, L, c_z], msa_mask [M, L],
    pair_mask [L, L]) -> (msa, pair)`` as FoldForge's graph calls it; :meth:`batched` takes a
    leading batch axis on every argument (``msa_mask [B, M, L]``, ``pair_mask [B, L, L]``)."""

    def __init__(self, c_msa: int = 64, c_pair: int = 128, n_heads_pair: int = 4, *, precision: str = "master",
                 masked_update: str = "compute") -> None:
        super().__init__()
        self.outer_product_mean = finish_op(OuterProductMean(c_msa, c_pair, 32, normalize_before_proj=False,
                                                             count_offset=OPM_COUNT_OFFSET), precision)
        self.msa_attention1 = finish_op(MSAPairWeightedAveraging(c_msa, c_pair, 8, None), precision)
        self.msa_transition = factories.transition(c_msa, 4, precision=precision)
        self.triangle_multiplication_outgoing = factories.triangle_multiplication(c_pair, outgoing=True,
                                                                                  precision=precision)
        self.triangle_multiplication_incoming = factories.triangle_multiplication(c_pair, outgoing=False,
                                                                                  precision=precision)
        self.pair_attention1 = factories.triangle_attention(c_pair, n_heads_pair, starting=True, model="af3",
                                                            precision=precision)
        self.pair_attention2 = factories.triangle_attention(c_pair, n_heads_pair, starting=False, model="af3",
                                                            precision=precision)
        self.pair_transition = factories.transition(c_pair, 4, precision=precision)
        for m in self.modules():
            if isinstance(m, _PairOp):
                m.masked_update = masked_update

    def forward(self, msa: torch.Tensor, pair: torch.Tensor, msa_mask: torch.Tensor, pair_mask: torch.Tensor):
        m, z = self.batched(msa[None], pair[None], msa_mask[None], pair_mask[None])
        return m[0], z[0]

    def batched(self, m: torch.Tensor, z: torch.Tensor, msa_mask: torch.Tensor, pair_mask: torch.Tensor):
        rows = msa_mask > 0
        columns = (msa_mask.amax(dim=1) > 0)  # a column is a key when any MSA row has it
        tokens = factories.token_mask(pair_mask)  # [B, L] from the pair mask's diagonal
        z = z + self.outer_product_mean(m, rows)
        m = self.msa_transition(self.msa_attention1(m, z, columns))
        z = self.triangle_multiplication_outgoing(z, tokens)
        z = self.triangle_multiplication_incoming(z, tokens)
        z = self.pair_attention1(z, tokens)
        z = self.pair_attention2(z, tokens)
        z = self.pair_transition(z)
        return m, z


def finish_op(module: nn.Module, precision: str) -> nn.Module:
    """An op module with the package's precision handling (fp32 masters under ``master``)."""
    return factories.finish(module, precision)
