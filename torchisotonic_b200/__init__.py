"""Batched isotonic regression for PyTorch on NVIDIA B200 (sm_100a): a drop-in for
``torchisotonic.isotonic`` over hand-written CUDA kernels behind a C ABI (include/tiso.h)."""

from torchisotonic_b200._api import isotonic, isotonic_varlen
from torchisotonic_b200.calibration import calibrate, fit_calibration
from torchisotonic_b200.soft_rank import soft_rank

__all__ = ["isotonic", "isotonic_varlen", "fit_calibration", "calibrate", "soft_rank"]
__version__ = "0.1.0"
