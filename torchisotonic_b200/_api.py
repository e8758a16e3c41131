"""Batched isotonic regression on B200: the drop-in for ``torchisotonic.isotonic``.

Same signature, validation, dtype rules, ``dim`` handling, NaN and empty-input semantics and
gradients as the reference (src/torchisotonic/_api.py:13-134); the fit, the clip, the casts
and the weight check run fused in the CUDA kernels of libtiso.so. CUDA tensors only: there is no
CPU path (use the reference, or the oracle in tests, on the CPU).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from torchisotonic_b200 import _ext, ops


def isotonic(
    y: Tensor,
    weight: Tensor | None = None,
    *,
    increasing: bool = True,
    y_min: float | None = None,
    y_max: float | None = None,
    dim: int = -1,
    exact: bool = True,
) -> Tensor:
    """Isotonic regression of every 1-D slice of ``y`` along ``dim``.

    For each slice, returns the non-decreasing (or, with ``increasing=False``,
    non-increasing) sequence closest to it in weighted least squares, like
    ``sklearn.isotonic.isotonic_regression``. ``weight`` must be positive and shaped like
    ``y`` (or broadcast to it). Results are clipped to ``[y_min, y_max]`` if given. A slice
    containing NaN comes back as NaN. Integer input becomes the default float dtype; float
    input keeps its dtype, with float16/bfloat16 computed in float32.

    Differentiable in ``y`` and ``weight``: the fit is constant on blocks of neighbouring
    elements, each the weighted mean of ``y`` over its block, so a gradient is averaged over
    the blocks.

    ``exact=False`` sums float32 data in float32 instead of float64: results within about 1e-3
    of the data's scale on hard inputs. It has no effect on float64.
    """
    if not isinstance(y, Tensor):
        raise TypeError(f"y must be a torch.Tensor, got {type(y).__name__}")
    if y.is_complex():
        raise TypeError("complex tensors are not supported")
    if y.ndim == 0:
        raise ValueError("y must have at least one dimension")
    out_dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
    acc = torch.float64 if out_dtype == torch.float64 else torch.float32
    # the slices along the last dimension already: no moves (nor their autograd nodes)
    last = dim == -1 or dim == y.ndim - 1
    rows = y if last else y.movedim(dim, -1)
    w: Tensor | None = None
    if weight is not None:
        if not isinstance(weight, Tensor):
            raise TypeError(f"weight must be a torch.Tensor, got {type(weight).__name__}")
        try:
            w = weight.to(device=y.device, dtype=acc)
            if w.shape != y.shape:
                w = w.broadcast_to(y.shape)
            if not last:
                w = w.movedim(dim, -1)
        except RuntimeError as e:
            raise ValueError(f"weight of shape {tuple(weight.shape)} does not fit y") from e
    shape = rows.shape
    if rows.numel() == 0:
        return y.to(out_dtype, copy=True)
    if not y.is_cuda:
        raise RuntimeError(
            "torchisotonic_b200 runs on CUDA tensors only (no CPU fallback); "
            "move y to a CUDA device"
        )
    if rows.dtype != out_dtype:  # integer input
        rows = rows.to(out_dtype)
    two_d = rows.ndim == 2
    flat_y = (rows if two_d else rows.reshape(-1, shape[-1])).contiguous()
    flat_w = None if w is None else (w if two_d else w.reshape(-1, shape[-1])).contiguous()
    lo = None if y_min is None else float(y_min)
    hi = None if y_max is None else float(y_max)
    if torch.compiler.is_compiling():
        # traced: the torchisotonic_b200::fit operator (fake kernel, registered autograd), which
        # the compiler keeps whole; eager calls take the same kernels with less host work
        need_grad = torch.is_grad_enabled() and (
            flat_y.requires_grad or (flat_w is not None and flat_w.requires_grad))
        out, _ = ops.fit(flat_y, flat_w, increasing, exact, need_grad, lo, hi)
    else:
        out = _Isotonic.apply(flat_y, flat_w, increasing, exact, lo, hi)
    if not two_d:
        out = out.reshape(shape)
    return out if last else out.movedim(-1, dim)


class _Isotonic(torch.autograd.Function):
    """The fit of [batch, n] rows, clipped, with its gradient averaged over its blocks (the
    reference's _Isotonic, src/torchisotonic/_api.py:73-97, with the clamp and the casts folded
    in); the eager twin of the torchisotonic_b200::fit operator and its registered autograd."""

    @staticmethod
    def forward(ctx: Any, flat_y: Tensor, flat_w: Tensor | None, increasing: bool, exact: bool,
                y_min: float | None, y_max: float | None) -> Tensor:
        need_grad = any(ctx.needs_input_grad[:2])
        # the weights checked first (one pass), the fit launched behind it; the host waits for
        # the check alone before raising or returning, while the fit runs
        check = None if flat_w is None else _ext.WeightCheck(flat_w)
        out, starts = _ext.isotonic_tiles(flat_y, flat_w, increasing, exact, need_grad,
                                          y_min, y_max, check and check.fused_flag)
        if check is not None and check.failed():
            raise ValueError("weight must be strictly positive")
        ctx.save_for_backward(flat_y, flat_w, starts)
        ctx.clip = (y_min, y_max)
        return out

    @staticmethod
    def backward(ctx: Any, grad: Tensor) -> tuple[Tensor | None, ...]:
        flat_y, flat_w, starts = ctx.saved_tensors
        want_y, want_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        y_min, y_max = ctx.clip
        need_y = want_w or y_min is not None or y_max is not None
        gy, gw = _ext.isotonic_grad(starts, grad.contiguous(), flat_w,
                                    flat_y if need_y else None, want_y, want_w, y_min, y_max)
        return gy, gw, None, None, None, None


def isotonic_varlen(
    values: Tensor,
    offsets: Tensor,
    weight: Tensor | None = None,
    *,
    increasing: bool = True,
    y_min: float | None = None,
    y_max: float | None = None,
    exact: bool = True,
    max_len: int | None = None,
) -> Tensor:
    """Isotonic regression of ragged rows laid end to end: row r is
    ``values[offsets[r]:offsets[r + 1]]``, each fitted on its own, as ``isotonic`` fits the rows
    of a batch (same dtype rules, clipping, NaN rows, ``exact`` and gradients in ``values`` and
    ``weight``). Returns the fits packed the same way.

    This replaces the padded batch that the reference's README describes for rows of unequal
    length (pad each row at its end past its maximum, fit, drop the padding): no padding is read
    or written. ``offsets``: 1-D integer tensor of ``batch + 1`` non-decreasing positions, on
    ``values``' device. ``max_len``: the longest row, at most 512 (computed from ``offsets``,
    with one synchronisation, when not given; a smaller value cuts longer rows). ``weight``:
    positive, shaped like ``values``.
    """
    if not isinstance(values, Tensor) or not isinstance(offsets, Tensor):
        raise TypeError("values and offsets must be torch.Tensors")
    if values.is_complex():
        raise TypeError("complex tensors are not supported")
    if values.ndim != 1 or offsets.ndim != 1 or offsets.numel() < 1:
        raise ValueError("values must be 1-D and offsets 1-D with at least one entry")
    if offsets.is_floating_point() or offsets.is_complex():
        raise TypeError("offsets must be an integer tensor")
    out_dtype = values.dtype if values.is_floating_point() else torch.get_default_dtype()
    acc = torch.float64 if out_dtype == torch.float64 else torch.float32
    if not values.is_cuda:
        raise RuntimeError(
            "torchisotonic_b200 runs on CUDA tensors only (no CPU fallback); "
            "move values to a CUDA device"
        )
    offsets = offsets.to(device=values.device, dtype=torch.int64).contiguous()
    w: Tensor | None = None
    if weight is not None:
        if not isinstance(weight, Tensor):
            raise TypeError(f"weight must be a torch.Tensor, got {type(weight).__name__}")
        try:
            w = weight.to(device=values.device, dtype=acc).broadcast_to(values.shape).contiguous()
        except RuntimeError as e:
            raise ValueError(f"weight of shape {tuple(weight.shape)} does not fit values") from e
    if max_len is None:
        lengths = offsets[1:] - offsets[:-1]
        max_len = int(lengths.max()) if lengths.numel() else 0
    if max_len > _ext.VARLEN_MAX:
        raise ValueError(f"ragged rows of more than {_ext.VARLEN_MAX} elements are not supported: "
                         "pad them into a batch for isotonic()")
    y = values if values.dtype == out_dtype else values.to(out_dtype)
    return _IsotonicVarlen.apply(y.contiguous(), w, offsets, int(max_len), increasing, exact,
                                 y_min, y_max)


class _IsotonicVarlen(torch.autograd.Function):
    """The fit of packed ragged rows, clipped, with its gradient averaged over its blocks."""

    @staticmethod
    def forward(ctx: Any, y: Tensor, w: Tensor | None, offsets: Tensor, max_len: int,
                increasing: bool, exact: bool, y_min: float | None,
                y_max: float | None) -> Tensor:
        need_grad = any(ctx.needs_input_grad[:2])
        check = None if w is None else _ext.WeightCheck(w)
        out, starts = _ext.isotonic_tiles_varlen(y, w, offsets, max_len, increasing, exact,
                                                 need_grad, y_min, y_max,
                                                 check and check.fused_flag)
        if check is not None and check.failed():
            raise ValueError("weight must be strictly positive")
        ctx.save_for_backward(y, w, offsets, starts)
        ctx.max_len = max_len
        ctx.clip = (y_min, y_max)
        return out

    @staticmethod
    def backward(ctx: Any, grad: Tensor) -> tuple[Tensor | None, ...]:
        y, w, offsets, starts = ctx.saved_tensors
        want_y, want_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        y_min, y_max = ctx.clip
        need_y = want_w or y_min is not None or y_max is not None
        gy, gw = _ext.isotonic_grad_varlen(starts, grad.contiguous(), w, y if need_y else None,
                                           offsets, ctx.max_len, want_y, want_w, y_min, y_max)
        return gy, gw, None, None, None, None, None, None
