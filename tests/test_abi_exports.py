"""The C-ABI library loads without a GPU and exports every entry point the header declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from foldforge_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "foldforge_b200.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|size_t)\s+(ffb_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_entry_points():
    assert set(declared()) == set(_lib.SIGNATURES)


def test_library_loads_and_exports_every_declared_symbol():
    if not _lib.LIBRARY.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(str(_lib.LIBRARY))
    for name in declared():
        assert hasattr(lib, name), name
    assert _lib.load().ffb_version() >= 100
