"""CPU oracle for the Pairformer pair-stack path. TEST INFRASTRUCTURE ONLY.

This package restates, in plain fp32/fp64 PyTorch on the CPU, the equations of
FoldForge's released-layout (legacy) ``PairformerBlock`` that the reference's own
parity test pins the engine ``pytorch`` backend to
(``tests/models/test_engine_graph.py:127-148``). Parameters use the ENGINE key schema
(the output of ``legacy/released.py:318-369``, ``pairformer_block_from_released``).

Who may use it: ``tests/`` (as the checker), ``__graft_entry__.smoke()`` (as the
checker) and ``bench.py`` (the ``cpu_baseline`` leg and ``--impl reference``). The
product package ``foldforge_b200`` never imports it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own legacy block (imported
from the reference tree in the build container) on seeded weights and inputs and commits
the outputs as fixtures; ``tests/test_oracle_golden.py`` checks this restatement against
them.
"""

from oracle.pairformer import (  # noqa: F401
    attention_pair_bias,
    block_flops,
    layer_norm,
    pairformer_block,
    rel_l2,
    transition,
    triangle_attention,
    triangle_multiplication,
)
