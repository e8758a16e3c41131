"""Builds torchisotonic_b200/libtiso.so: the CUDA kernels behind include/tiso.h, for sm_100a.

    python -m torchisotonic_b200.build [--verbose]

nvcc compiles for the B200 (compute_100a / sm_100a) only; no JIT build at import time.
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
LIB = PKG / "libtiso.so"
SOURCES = [CSRC / "tiso.cu", CSRC / "calib.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "tiso.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []),
           "-o", str(tmp), *map(str, SOURCES), "-lcudart"]
    subprocess.run(cmd, check=True, cwd=str(ROOT))
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
