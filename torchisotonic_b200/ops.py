"""The operator layer as torch custom operators (torch.library), over the C ABI of libtiso.so.

Two operators keep the reference's schemas (src/torchisotonic/csrc/ops.cpp:47-50), so that code
calling ``torch.ops.torchisotonic.isotonic_tiles`` / ``isotonic_grad`` can call
``torch.ops.torchisotonic_b200.*`` with the same arguments:

* ``isotonic_tiles(Tensor y, Tensor? w, bool increasing, bool exact=True, bool with_starts=False)
  -> Tensor[]``: ``[out, starts]``, starts empty unless ``with_starts``;
* ``isotonic_grad(Tensor out, Tensor starts, Tensor g, Tensor? w, Tensor? y) -> Tensor[]``:
  ``[grad_y, grad_w]``, grad_w empty when y is None. ``out`` is not read: the kernel recomputes
  each block's mean from y and w where d/dw needs it.

Two more carry what this library folds into its kernels, and are what ``isotonic()`` runs:

* ``fit(Tensor y, Tensor? w, bool increasing, bool exact, bool with_starts, float? y_min,
  float? y_max) -> (Tensor, Tensor)``: the clipped fit in y's dtype (float16 and bfloat16 read
  as they are) and its block starts; raises ValueError when a weight is not positive (one pass
  over the weights ahead of the fit; its flag is read inside the operator);
* ``fit_grad(Tensor starts, Tensor g, Tensor? w, Tensor? y, bool want_y, bool want_w,
  float? y_min, float? y_max) -> (Tensor, Tensor)``: d/dy and d/dw (empty when not wanted),
  the clamp's inclusive mask applied.

``fit`` has its autograd registered (the reference's _Isotonic, src/torchisotonic/_api.py:73-97)
and every operator a fake (meta) implementation, so ``torch.compile`` traces through them
without a graph break. There is no CPU kernel: CUDA tensors only.
"""

from __future__ import annotations

import torch
from torch import Tensor

from torchisotonic_b200 import _ext

_NS = "torchisotonic_b200"


def _acc(dtype: torch.dtype) -> torch.dtype:
    return _ext.acc_dtype(dtype)


# ---------------------------------------------------------------------------------------------
# The reference's schemas


@torch.library.custom_op(
    f"{_NS}::isotonic_tiles", mutates_args=(),
    schema="(Tensor y, Tensor? w, bool increasing, bool exact=True, bool with_starts=False)"
           " -> Tensor[]")
def isotonic_tiles(y: Tensor, w: Tensor | None, increasing: bool, exact: bool = True,
                   with_starts: bool = False) -> list[Tensor]:
    out, starts = _ext.isotonic_tiles(y, w, increasing, exact, with_starts)
    return [out, starts]


@isotonic_tiles.register_fake
def _(y, w, increasing, exact=True, with_starts=False):
    starts = y.new_empty(y.shape if with_starts else (0,), dtype=torch.bool)
    return [torch.empty_like(y), starts]


@torch.library.custom_op(
    f"{_NS}::isotonic_grad", mutates_args=(),
    schema="(Tensor out, Tensor starts, Tensor g, Tensor? w, Tensor? y) -> Tensor[]")
def isotonic_grad(out: Tensor, starts: Tensor, g: Tensor, w: Tensor | None,
                  y: Tensor | None) -> list[Tensor]:
    want_w = y is not None and w is not None
    gy, gw = _ext.isotonic_grad(starts, g.contiguous(), w, y if want_w else None, True, want_w)
    if gw is None:
        gw = g.new_empty((0,), dtype=_acc(g.dtype))
    return [gy, gw]


@isotonic_grad.register_fake
def _(out, starts, g, w, y):
    gw = (torch.empty(g.shape, dtype=_acc(g.dtype), device=g.device)
          if (y is not None and w is not None) else g.new_empty((0,), dtype=_acc(g.dtype)))
    return [torch.empty_like(g), gw]


# ---------------------------------------------------------------------------------------------
# The fused operators behind isotonic()


@torch.library.custom_op(f"{_NS}::fit", mutates_args=())
def fit(y: Tensor, w: Tensor | None, increasing: bool, exact: bool, with_starts: bool,
        y_min: float | None, y_max: float | None) -> tuple[Tensor, Tensor]:
    check = None if w is None else _ext.WeightCheck(w)
    out, starts = _ext.isotonic_tiles(y, w, increasing, exact, with_starts, y_min, y_max,
                                      check and check.fused_flag)
    if check is not None and check.failed():
        raise ValueError("weight must be strictly positive")
    return out, starts


@fit.register_fake
def _(y, w, increasing, exact, with_starts, y_min, y_max):
    return torch.empty_like(y), y.new_empty(y.shape if with_starts else (0,), dtype=torch.bool)


@torch.library.custom_op(f"{_NS}::fit_grad", mutates_args=())
def fit_grad(starts: Tensor, g: Tensor, w: Tensor | None, y: Tensor | None, want_y: bool,
             want_w: bool, y_min: float | None, y_max: float | None) -> tuple[Tensor, Tensor]:
    gy, gw = _ext.isotonic_grad(starts, g.contiguous(), w, y, want_y, want_w, y_min, y_max)
    if gy is None:
        gy = g.new_empty((0,))
    if gw is None:
        gw = g.new_empty((0,), dtype=_acc(g.dtype))
    return gy, gw


@fit_grad.register_fake
def _(starts, g, w, y, want_y, want_w, y_min, y_max):
    gy = torch.empty_like(g) if want_y else g.new_empty((0,))
    gw = (torch.empty(g.shape, dtype=_acc(g.dtype), device=g.device) if want_w
          else g.new_empty((0,), dtype=_acc(g.dtype)))
    return gy, gw


def _fit_setup(ctx, inputs, output) -> None:
    y, w, _increasing, _exact, _with_starts, y_min, y_max = inputs
    _, starts = output
    ctx.save_for_backward(y, w, starts)
    ctx.clip = (y_min, y_max)


def _fit_backward(ctx, grad_out: Tensor, _grad_starts: Tensor):
    y, w, starts = ctx.saved_tensors
    want_y, want_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    y_min, y_max = ctx.clip
    need_y = want_w or y_min is not None or y_max is not None
    gy, gw = fit_grad(starts, grad_out, w, y if need_y else None, want_y, want_w, y_min, y_max)
    return (gy if want_y else None, gw if want_w else None, None, None, None, None, None)


torch.library.register_autograd(f"{_NS}::fit", _fit_backward, setup_context=_fit_setup)
