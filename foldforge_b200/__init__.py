"""B200-native (sm_100a) backend of FoldForge's Pairformer pair stack.

* :mod:`foldforge_b200.engine` -- the engine-module contract FoldForge's graph consumes
  (op classes with ``pytorch`` / ``b200`` backends, backend plan, guard, observations,
  ``run_block``).
* :mod:`foldforge_b200.kernels` -- torch-facing wrappers of the C ABI
  (``include/foldforge_b200.h``) implemented by ``_ffb.so``.
* :func:`load` -- the path's share of ``foldforge.load(..., backend=...)``
  (``src/foldforge/models/__init__.py:134-148``): a Pairformer trunk from engine-key block
  state dicts, configured for a precision and given its backends by a plan.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

import torch

__version__ = "0.1.0"


def load(
    blocks: Sequence[Mapping[str, torch.Tensor]],
    *,
    backend: str = "miniworld",
    engine_ops: Mapping[str, str] | None = None,
    unsupported: str = "fallback",
    dtype: torch.dtype = torch.bfloat16,
    device: str | torch.device = "cuda",
    masked_update: str = "zero",
    d_single: int = 384,
):
    """A ``Pairformer`` trunk of ``len(blocks)`` AF3 blocks loaded strictly from ``blocks``
    (engine state-dict keys), moved to ``device`` with fp32 parameters, precision from
    ``dtype`` (bf16 -> master, fp32 -> fp32) and backends from
    ``BackendPlan.make(backend, engine_ops, unsupported)``. The plan and per-module choices
    are in ``trunk.foldforge_load_report``."""
    from foldforge_b200.engine.backends import BackendPlan
    from foldforge_b200.engine.configure import configure_model
    from foldforge_b200.engine.factories import finish
    from foldforge_b200.engine.install import install_engine
    from foldforge_b200.engine.modules import Pairformer, PairformerConfig

    plan = BackendPlan.make(backend, engine_ops, unsupported)
    config = PairformerConfig(d_single=d_single, masked_update=masked_update)
    trunk = finish(Pairformer(config, len(blocks)), "master" if dtype == torch.bfloat16 else "fp32")
    for block, state in zip(trunk.blocks, blocks, strict=True):
        block.load_state_dict(state, strict=True)
    configure_model(trunk, backend, dtype, device)
    install_engine(trunk, device, plan=plan)
    return trunk
