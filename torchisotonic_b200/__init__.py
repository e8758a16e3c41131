"""Batched isotonic regression for PyTorch on NVIDIA B200 (sm_100a): a drop-in for
``torchisotonic.isotonic`` over hand-written CUDA kernels behind a C ABI (include/tiso.h)."""

from torchisotonic_b200._api import isotonic
from torchisotonic_b200.calibration import calibrate, fit_calibration

__all__ = ["isotonic", "fit_calibration", "calibrate"]
__version__ = "0.1.0"
