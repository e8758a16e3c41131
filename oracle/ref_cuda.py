"""TEST AND BENCH INFRASTRUCTURE ONLY - the reference's own CUDA operators, built from its sources.

The reference compiles its operators on first use (src/torchisotonic/_ext.py:53-67):
``torch.utils.cpp_extension.load`` of ``csrc/ops.cpp`` and ``csrc/ops_tiles.cu`` with ``-O3``,
registering ``torch.ops.torchisotonic.{isotonic, isotonic_tiles, isotonic_grad}``
(``ops.cpp:45-51``, ``ops_tiles.cu:8-11``). This script runs the same load with the same
sources and flags, unmodified, for the B200 (``TORCH_CUDA_ARCH_LIST=10.0``: there is no GPU
where it is built to take the architecture from), into ``oracle/_ref/ref_cuda/``. That folder
is not in git; it travels with the working tree to the GPU machine, where ``load()`` registers
the prebuilt operators without compiling anything.

    python oracle/ref_cuda.py /path/to/torchisotonic-checkout

Only ``bench.py`` (its comparison with the reference's GPU operator) and ``tests/`` may load
it; nothing in the package does.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "_ref" / "ref_cuda"
NAME = "torchisotonic_ops"
LIB = OUT / f"{NAME}.so"


def build(ref: str | Path) -> Path:
    """Compiles the reference's ops.cpp and ops_tiles.cu into ``LIB`` (as its _ext._load does)."""
    csrc = Path(ref) / "src" / "torchisotonic" / "csrc"
    if not (csrc / "ops_tiles.cu").exists():
        raise FileNotFoundError(f"no reference checkout at {ref}")
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils import cpp_extension

    OUT.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name=NAME,
        sources=[str(csrc / "ops.cpp"), str(csrc / "ops_tiles.cu")],
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3"],
        build_directory=str(OUT),
        is_python_module=False,
        verbose=False,
    )
    return LIB


_loaded = False


def load():
    """``torch.ops.torchisotonic`` from the prebuilt library, or None where it was not built."""
    global _loaded
    import torch

    if not _loaded:
        if not LIB.exists():
            return None
        torch.ops.load_library(str(LIB))
        _loaded = True
    return torch.ops.torchisotonic


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/torchisotonic-checkout")
    print(build(sys.argv[1]))
