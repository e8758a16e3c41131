"""Batched isotonic regression for PyTorch on NVIDIA B200 (sm_100a): a drop-in for
``torchisotonic.isotonic`` over hand-written CUDA kernels behind a C ABI (include/tiso.h)."""

from torchisotonic_b200._api import isotonic

__all__ = ["isotonic"]
__version__ = "0.1.0"
