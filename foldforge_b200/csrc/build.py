"""Build ``foldforge_b200/_ffb.so`` from the CUDA sources with nvcc for sm_100a only.

``python -m foldforge_b200.csrc.build`` (or ``__graft_entry__.build()``). The library is
built in-tree so it travels with the repository snapshot; nvcc cross-compiles without a
GPU. Each translation unit is compiled to an object in ``_build/`` and relinked only when
a source or header changed.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
OUT = PKG / "_ffb.so"
BUILD = PKG.parent / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def sources() -> list[Path]:
    return sorted(HERE.glob("*.cu"))


def _newest_header() -> float:
    hs = list(HERE.glob("*.h")) + list(HERE.glob("*.cuh")) + list((PKG.parent / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(verbose: bool = False) -> Path:
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    BUILD.mkdir(exist_ok=True)
    objs = []
    header_time = _newest_header()
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, header_time):
            continue
        cmd = [nvcc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        log = BUILD / (src.stem + ".ptxas.txt")
        log.write_text(res.stdout + res.stderr)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed on {src.name}")
        if verbose:
            sys.stderr.write(res.stderr)
    if not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(OUT), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("nvcc link failed")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
