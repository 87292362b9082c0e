"""Build libsolattn.so in-tree with nvcc for sm_100a (no JIT, no torch extension).

``python -m sol_attn_b200.build`` (or ``build()``) compiles every ``csrc/*.cu`` into one
shared library next to this file.  The library is rebuilt only when a source or header is
newer than it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parents[1] / "include"
LIB = PKG / "libsolattn.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = shutil.which("nvcc") or os.path.join(cuda, "bin", "nvcc")
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")))
    return newest > LIB.stat().st_mtime


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> Path:
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *extra_flags, "-I", str(INCLUDE), "-o", str(tmp),
           *map(str, sources())]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [])
