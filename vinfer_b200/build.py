"""Build the in-tree CUDA library ``vinfer_b200/libvinfer_sampler.so`` for sm_100a.

The library is plain C ABI (``include/vinfer_sampler.h``) compiled by nvcc; nothing here
depends on torch. ``python -m vinfer_b200.build`` (or ``__graft_entry__.build()``) rebuilds it
when a source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libvinfer_sampler.so"
SOURCES = [CSRC / "sampler.cu"]
HEADERS = [INCLUDE / "vinfer_sampler.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: the sampler library cannot be built")
    return cand


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources; return its path."""
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", "-shared", "-o", str(tmp),
           *map(str, SOURCES), "-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
