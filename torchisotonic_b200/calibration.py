"""Calibration curves around the fit: the steps the reference gives as torch code next to
``isotonic`` (README.md:43-56, "Calibrating a classifier"; examples/ctr_calibration/
calibrate.py:163-186), here on the CUDA kernels of libtiso.so.

``fit_calibration(scores, labels)`` is scikit-learn's ``IsotonicRegression`` curve: the pairs
sorted by score, equal scores pooled into their mean label weighted by their count, then the
increasing isotonic fit of those means. The reference does the pre-step with ``torch.sort``,
``unique_consecutive``, ``index_add_`` and a division; here it is one radix sort of the pairs
and three passes over them (``tiso_calib_groups``), then the same fit as ``isotonic``.
``calibrate(new_scores, xs, fit)`` reads scores on the curve: ``torch.searchsorted``, the
clamps and the linear interpolation of the reference, fused into one kernel
(``tiso_calib_interp``) with torch's roundings.
"""

from __future__ import annotations

import torch
from torch import Tensor

from torchisotonic_b200 import _ext

_SMALL_LABELS = (torch.bool, torch.uint8, torch.int8, torch.int16, torch.float16,
                 torch.bfloat16, torch.float32)


def _key_dtype(dtype: torch.dtype) -> torch.dtype:
    if dtype == torch.float64 or not (dtype.is_floating_point or dtype == torch.bool):
        return torch.float64  # integers: exact up to 2**53
    return torch.float32


def fit_calibration(scores: Tensor, labels: Tensor) -> tuple[Tensor, Tensor]:
    """The calibration curve of ``labels`` over ``scores`` (1-D CUDA tensors of one length),
    as scikit-learn's ``IsotonicRegression`` fits it, equal scores pooled into their mean:
    returns ``(xs, fit)``, the distinct scores in increasing order (in the scores' dtype) and
    the non-decreasing fit at each (float64). The reference's ``fit_calibration``
    (README.md:43-50).

    Sums of labels are float64, in a fixed order (the result does not vary between runs).
    Raises ValueError for a NaN score; a NaN label makes the whole fit NaN, as ``isotonic``
    does for a row holding NaN. Of equal scores -0.0 and 0.0, ``xs`` keeps -0.0.
    """
    if not isinstance(scores, Tensor) or not isinstance(labels, Tensor):
        raise TypeError("scores and labels must be torch.Tensors")
    if scores.is_complex() or labels.is_complex():
        raise TypeError("complex tensors are not supported")
    if scores.dim() != 1 or labels.dim() != 1 or scores.numel() != labels.numel():
        raise ValueError("scores and labels must be 1-D tensors of one length")
    if scores.numel() == 0:
        return scores.clone(), torch.empty(0, dtype=torch.float64, device=scores.device)
    if not scores.is_cuda:
        raise RuntimeError(
            "torchisotonic_b200 runs on CUDA tensors only (no CPU fallback); "
            "move scores to a CUDA device"
        )
    keys = scores.to(_key_dtype(scores.dtype)).contiguous()
    lab_dtype = torch.float32 if labels.dtype in _SMALL_LABELS else torch.float64
    labs = labels.to(device=scores.device, dtype=lab_dtype).contiguous()
    xs, y, w, groups = _ext.calib_groups(keys, labs)
    g, nan = groups.tolist()
    if nan:
        raise ValueError("scores must not be NaN")
    fit, _ = _ext.isotonic_tiles(y[:g][None], w[:g][None], increasing=True, exact=True)
    return xs[:g].to(scores.dtype), fit[0]


def calibrate(new_scores: Tensor, xs: Tensor, fit: Tensor) -> Tensor:
    """Calibrated values of ``new_scores`` on the curve ``(xs, fit)`` of ``fit_calibration``:
    linear between its points, constant beyond them; NaN scores read the last point's value
    (``searchsorted`` puts them past the end). The reference's ``calibrate`` (README.md:53-56),
    every step rounded as torch rounds it, in the scores' dtype up to ``t`` and in float64
    from there (float16 and bfloat16 scores are computed in float32). Returns the shape of
    ``new_scores`` in the dtype torch's expression gives (float64 for a float64 ``fit``).
    """
    if not isinstance(new_scores, Tensor) or not isinstance(xs, Tensor) \
            or not isinstance(fit, Tensor):
        raise TypeError("new_scores, xs and fit must be torch.Tensors")
    if xs.dim() != 1 or fit.dim() != 1 or xs.numel() != fit.numel() or xs.numel() == 0:
        raise ValueError("xs and fit must be 1-D tensors of one length >= 1")
    if not new_scores.is_cuda:
        raise RuntimeError(
            "torchisotonic_b200 runs on CUDA tensors only (no CPU fallback); "
            "move new_scores to a CUDA device"
        )
    key = torch.float64 if new_scores.dtype == torch.float64 else torch.float32
    if not new_scores.dtype.is_floating_point:
        raise TypeError("new_scores must be a floating-point tensor")
    out_dtype = torch.promote_types(fit.dtype, new_scores.dtype)
    x = new_scores.to(key).contiguous().view(-1)
    pts = xs.to(device=new_scores.device, dtype=key).contiguous()
    f = fit.to(device=new_scores.device, dtype=torch.float64).contiguous()
    out = _ext.calib_interp(x, pts, f)
    return out.view(new_scores.shape).to(out_dtype)
