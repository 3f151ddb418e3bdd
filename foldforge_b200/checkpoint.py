"""Reading FoldForge's miniworld-format checkpoints for the pair stack.

A miniworld file (``src/foldforge/models/checkpoints/miniworld.py:1-30``) is a ``torch.save``
dict ``{"format": "miniworld", "version": 1, "family": ..., "source": ..., "state_dict":
{name: fp32 tensor}}`` whose keys are the FoldForge graph's engine-class keys, read with
``weights_only=True``. In the AF3 graph the pair stack's blocks sit at
``evoformer.trunk_pairformer.<i>.`` (the Pairformer trunk, ``models/architectures/af3.py:245``)
and ``evoformer.msa_stack.<i>.`` (the MSA stack, ``af3.py:214-233``), with exactly the keys
this package's :class:`~foldforge_b200.engine.modules.PairformerBlock` and
:class:`~foldforge_b200.engine.evoformer.EvoformerBlock` carry. This module reads such a file
with the reference's checks (format tag, version, family: ``miniworld.py:96-131``), takes the
blocks of the requested stack by prefix, and loads them STRICTLY (a missing, extra or
mis-shaped key is an error) into a trunk or an MSA stack on the ``b200`` backend.
"""

from __future__ import annotations

import re
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch

FORMAT = "miniworld"
VERSION = 1
SUFFIX = ".miniworld.pt"
#: Key prefixes of the pair-stack blocks in the AF3 graph.
TRUNK_PREFIX = "evoformer.trunk_pairformer"
MSA_PREFIX = "evoformer.msa_stack"


def is_native(path: str | Path) -> bool:
    """Whether ``path`` names a miniworld-format file (by suffix)."""
    return Path(path).name.endswith(SUFFIX)


def read(path: str | Path) -> dict[str, Any]:
    """The checked contents of a miniworld-format file (``weights_only`` load; the format tag
    and version verified; ``ValueError`` otherwise)."""
    path = Path(path)
    blob = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(blob, dict) or blob.get("format") != FORMAT:
        tag = blob.get("format") if isinstance(blob, dict) else None
        raise ValueError(f"{path} is not a miniworld-format checkpoint (format tag {tag!r})")
    if blob.get("version") != VERSION:
        raise ValueError(f"{path} is miniworld format version {blob.get('version')}; this code reads version "
                         f"{VERSION}. Convert the release again.")
    if not isinstance(blob.get("state_dict"), Mapping):
        raise ValueError(f"{path} has no state_dict")
    return blob


def write(path: str | Path, state_dict: Mapping[str, torch.Tensor], *, family: str, source: str | None = None) -> None:
    """Write ``state_dict`` (fp32) in the miniworld format (the layout ``read`` checks)."""
    blob = {"format": FORMAT, "version": VERSION, "family": family, "source": source,
            "state_dict": {k: v.detach().to("cpu", torch.float32).contiguous() for k, v in state_dict.items()}}
    torch.save(blob, Path(path))


def block_states(state_dict: Mapping[str, torch.Tensor], prefix: str) -> list[dict[str, torch.Tensor]]:
    """The per-block state dicts under ``<prefix>.<i>.``, in block order; the indices must run
    0..n-1 without a gap (``ValueError`` otherwise; ``[]`` when no key has the prefix)."""
    pattern = re.compile(re.escape(prefix) + r"\.(\d+)\.(.+)")
    blocks: dict[int, dict[str, torch.Tensor]] = {}
    for key, value in state_dict.items():
        m = pattern.fullmatch(key)
        if m:
            blocks.setdefault(int(m.group(1)), {})[m.group(2)] = value
    if sorted(blocks) != list(range(len(blocks))):
        raise ValueError(f"{prefix}: block indices {sorted(blocks)} are not 0..{len(blocks) - 1}")
    return [blocks[i] for i in range(len(blocks))]


def _checked(path: str | Path, family: str | None) -> Mapping[str, torch.Tensor]:
    blob = read(path)
    if family is not None and blob.get("family") != family:
        raise ValueError(f"{path} holds family {blob.get('family')!r}, the model is {family!r}")
    return blob["state_dict"]


def load_trunk(path: str | Path, *, family: str | None = "alphafold3", prefix: str = TRUNK_PREFIX,
               **load_kwargs: Any):
    """The Pairformer trunk of a miniworld file as a :class:`Pairformer` of this package
    (:func:`foldforge_b200.load` with ``load_kwargs``: backend, dtype, device ...). Raises
    ``ValueError`` when the file holds no block under ``prefix``."""
    import foldforge_b200

    states = block_states(_checked(path, family), prefix)
    if not states:
        raise ValueError(f"{path} has no {prefix}.<i>.* keys")
    return foldforge_b200.load(states, **load_kwargs)


def load_msa_stack(path: str | Path, *, family: str | None = "alphafold3", prefix: str = MSA_PREFIX,
                   backend: str = "miniworld", dtype: torch.dtype = torch.bfloat16,
                   device: str | torch.device = "cuda", c_msa: int = 64, c_pair: int = 128,
                   n_heads_pair: int = 4) -> torch.nn.ModuleList:
    """The MSA stack of a miniworld file as :class:`EvoformerBlock` s of this package (AF3
    widths by default), loaded strictly, moved to ``device`` and given their backends."""
    from foldforge_b200.engine.backends import BackendPlan
    from foldforge_b200.engine.configure import configure_model
    from foldforge_b200.engine.evoformer import EvoformerBlock
    from foldforge_b200.engine.install import install_engine

    states = block_states(_checked(path, family), prefix)
    if not states:
        raise ValueError(f"{path} has no {prefix}.<i>.* keys")
    precision = "master" if dtype == torch.bfloat16 else "fp32"
    stack = torch.nn.ModuleList(EvoformerBlock(c_msa, c_pair, n_heads_pair, precision=precision) for _ in states)
    for block, state in zip(stack, states, strict=True):
        block.load_state_dict(state, strict=True)
    configure_model(stack, backend, dtype, device)
    install_engine(stack, device, plan=BackendPlan.make(backend))
    return stack


__all__ = ["FORMAT", "MSA_PREFIX", "SUFFIX", "TRUNK_PREFIX", "VERSION", "block_states", "is_native", "load_msa_stack",
           "load_trunk", "read", "write"]
