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

from torchisotonic_b200 import _ext


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
    rows = y.movedim(dim, -1)
    w: Tensor | None = None
    if weight is not None:
        if not isinstance(weight, Tensor):
            raise TypeError(f"weight must be a torch.Tensor, got {type(weight).__name__}")
        try:
            w = weight.to(device=y.device, dtype=acc).broadcast_to(y.shape).movedim(dim, -1)
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
    flat_y = rows.reshape(-1, shape[-1]).contiguous()
    flat_w = None if w is None else w.reshape(-1, shape[-1]).contiguous()
    out: Tensor = _Isotonic.apply(flat_y, flat_w, increasing, exact, y_min, y_max)
    return out.reshape(shape).movedim(-1, dim)


class _Isotonic(torch.autograd.Function):
    """The fit of [batch, n] rows, clipped, with its gradient: averaging over its blocks
    (the reference's _Isotonic, src/torchisotonic/_api.py:73-97, with the clamp and the
    casts folded in)."""

    @staticmethod
    def forward(
        ctx: Any,
        flat_y: Tensor,
        flat_w: Tensor | None,
        increasing: bool,
        exact: bool,
        y_min: float | None,
        y_max: float | None,
    ) -> Tensor:
        need_grad = any(ctx.needs_input_grad[:2])
        bad = None
        if flat_w is not None:
            bad = torch.empty(1, dtype=torch.int32, device=flat_y.device)
        out, starts = _ext.isotonic_tiles(flat_y, flat_w, increasing, exact, need_grad,
                                          y_min, y_max, bad)
        if bad is not None and bool(bad.item()):
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
