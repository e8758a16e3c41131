"""TEST INFRASTRUCTURE ONLY - the CPU oracle for torchisotonic_b200.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use this
package, and only as the checker (or the timed CPU baseline), never as the product path.

It wraps two shared libraries built by ``oracle/Makefile``:

* ``liboracle.so`` (``pava.c``): a plain-C restatement of torchisotonic's CPU solver
  (``src/torchisotonic/csrc/pava.h:16-69``), its decreasing/clip handling
  (``src/torchisotonic/_api.py:68-69,131-134``) and its CPU backward (``_api.py:86-115``), in
  the reference's own precision (bit-exact with the reference CPU op) or in extended precision
  (the exact block partition, the bar for the GPU kernels).
* ``_ref/libpava_ref.so``: the reference's own ``pava.h`` compiled here (present only where the
  reference checkout was available at build time); its rows run in parallel like
  ``src/torchisotonic/csrc/ops.cpp:30``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PREC_REFERENCE = 0
PREC_EXTENDED = 1

_lib: ctypes.CDLL | None = None
_ref: ctypes.CDLL | None = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_dbl = ctypes.c_double


def build() -> None:
    """Compiles the oracle (and the reference's solver, when the checkout is present)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        _lib = ctypes.CDLL(str(path))
        for name in ("oracle_fit_f32", "oracle_fit_f64"):
            f = getattr(_lib, name)
            f.argtypes = [_p, _p, _p, _p, _i64, _i64, _int, _int, _int, _int, _dbl, _dbl, _int]
            f.restype = _int
        for name in ("oracle_grad_f32", "oracle_grad_f64"):
            f = getattr(_lib, name)
            f.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _int, _dbl, _dbl, _int]
            f.restype = _int
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own CPU solver, or None where it was not built."""
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libpava_ref.so"
        if not path.exists():
            return None
        _ref = ctypes.CDLL(str(path))
        for name in ("ref_fit_f32", "ref_fit_f64"):
            f = getattr(_ref, name)
            f.argtypes = [_p, _p, _p, _p, _i64, _i64, _int, _int]
            f.restype = _int
        _ref.ref_max_threads.restype = _int
    return _ref


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def _rows(y: np.ndarray, w: np.ndarray | None) -> tuple[np.ndarray, np.ndarray | None]:
    if y.dtype not in (np.float32, np.float64):
        raise TypeError(f"oracle rows must be float32 or float64, got {y.dtype}")
    y2 = np.ascontiguousarray(y.reshape(-1, y.shape[-1]))
    w2 = None
    if w is not None:
        w2 = np.ascontiguousarray(np.broadcast_to(w, y.shape).astype(y.dtype).reshape(y2.shape))
    return y2, w2


def fit(
    y: np.ndarray,
    w: np.ndarray | None = None,
    *,
    increasing: bool = True,
    y_min: float | None = None,
    y_max: float | None = None,
    precision: int = PREC_EXTENDED,
    threads: int = 0,
) -> tuple[np.ndarray, np.ndarray]:
    """The isotonic fit of every row (last axis) of y, clipped, and where its blocks start."""
    y2, w2 = _rows(y, w)
    batch, n = y2.shape
    out = np.empty_like(y2)
    starts = np.empty(y2.shape, dtype=np.uint8)
    f = lib().oracle_fit_f32 if y2.dtype == np.float32 else lib().oracle_fit_f64
    rc = f(_ptr(y2), _ptr(w2), _ptr(out), _ptr(starts), batch, n, int(increasing), precision,
           int(y_min is not None), int(y_max is not None),
           0.0 if y_min is None else float(y_min), 0.0 if y_max is None else float(y_max),
           threads)
    if rc:
        raise RuntimeError(f"oracle fit failed ({rc})")
    return out.reshape(y.shape), starts.astype(bool).reshape(y.shape)


def grad(
    fit_: np.ndarray,
    starts: np.ndarray,
    g: np.ndarray,
    w: np.ndarray | None = None,
    y: np.ndarray | None = None,
    *,
    y_min: float | None = None,
    y_max: float | None = None,
    threads: int = 0,
) -> tuple[np.ndarray, np.ndarray | None]:
    """Gradients of the (clipped) fit in y and, given y, in w, from the blocks in ``starts``."""
    dt = fit_.dtype
    shape = fit_.shape
    n = shape[-1]
    f2 = np.ascontiguousarray(fit_.reshape(-1, n))
    s2 = np.ascontiguousarray(starts.reshape(-1, n).astype(np.uint8))
    g2 = np.ascontiguousarray(g.reshape(-1, n).astype(dt))
    w2 = None if w is None else np.ascontiguousarray(np.broadcast_to(w, shape).astype(dt).reshape(-1, n))
    y2 = None if y is None else np.ascontiguousarray(y.reshape(-1, n).astype(dt))
    gy = np.empty_like(f2)
    gw = np.empty_like(f2) if y is not None else None
    f = lib().oracle_grad_f32 if dt == np.float32 else lib().oracle_grad_f64
    rc = f(_ptr(f2), _ptr(s2), _ptr(g2), _ptr(w2), _ptr(y2), _ptr(gy), _ptr(gw), f2.shape[0], n,
           int(y_min is not None), int(y_max is not None),
           0.0 if y_min is None else float(y_min), 0.0 if y_max is None else float(y_max),
           threads)
    if rc:
        raise RuntimeError(f"oracle grad failed ({rc})")
    return gy.reshape(shape), None if gw is None else gw.reshape(shape)


def ref_fit(
    y: np.ndarray, w: np.ndarray | None = None, *, increasing: bool = True, threads: int = 0
) -> tuple[np.ndarray, np.ndarray]:
    """The reference's own CPU solver (compiled from its pava.h), unclipped."""
    r = ref_lib()
    if r is None:
        raise RuntimeError("oracle/_ref/libpava_ref.so was not built (no reference checkout)")
    y2, w2 = _rows(y, w)
    batch, n = y2.shape
    out = np.empty_like(y2)
    starts = np.empty(y2.shape, dtype=np.uint8)
    f = r.ref_fit_f32 if y2.dtype == np.float32 else r.ref_fit_f64
    if f(_ptr(y2), _ptr(w2), _ptr(out), _ptr(starts), batch, n, int(increasing), threads):
        raise RuntimeError("reference fit failed")
    return out.reshape(y.shape), starts.astype(bool).reshape(y.shape)


def cpu_threads() -> int:
    return os.cpu_count() or 1


def isotonic(y, weight=None, *, increasing=True, y_min=None, y_max=None, dim=-1,
             precision: int = PREC_EXTENDED, with_starts: bool = False, threads: int = 0):
    """The oracle behind torchisotonic.isotonic's semantics (src/torchisotonic/_api.py:43-70):
    integer input becomes the default float dtype, float16/bfloat16 are computed in float32,
    the fit runs along ``dim`` and is clipped, then cast back. Takes and returns CPU torch
    tensors; with ``with_starts`` also returns the [batch, n] block starts."""
    import torch

    out_dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
    acc = torch.float64 if out_dtype == torch.float64 else torch.float32
    rows = y.movedim(dim, -1)
    shape = rows.shape
    if rows.numel() == 0:
        res = y.to(out_dtype, copy=True)
        return (res, torch.zeros(0, dtype=torch.bool)) if with_starts else res
    flat_y = rows.reshape(-1, shape[-1]).to(acc).contiguous().numpy()
    flat_w = None
    if weight is not None:
        flat_w = (weight.to(acc).broadcast_to(y.shape).movedim(dim, -1)
                  .reshape(flat_y.shape).contiguous().numpy())
    out, starts = fit(flat_y, flat_w, increasing=increasing, y_min=y_min, y_max=y_max,
                      precision=precision, threads=threads)
    res = torch.from_numpy(out).reshape(shape).movedim(-1, dim).to(out_dtype)
    if with_starts:
        return res, torch.from_numpy(starts)
    return res


def fit_calibration(scores: np.ndarray, labels: np.ndarray, precision: int = PREC_EXTENDED):
    """The calibration curve of the reference's recipe (README.md:43-50: sort, pool equal scores
    into their mean label weighted by their count, increasing isotonic fit), in numpy with the
    oracle's fit: returns (xs, fit float64). Labels are summed in float64 in sorted order."""
    order = np.argsort(scores, kind="stable")
    s = scores[order]
    lab = labels[order].astype(np.float64)
    head = np.ones(s.size, dtype=bool)
    head[1:] = s[1:] != s[:-1]
    first = np.flatnonzero(head)
    counts = np.diff(np.append(first, s.size)).astype(np.float64)
    sums = np.add.reduceat(lab, first)
    out, _ = fit((sums / counts)[None], counts[None], increasing=True, precision=precision)
    return s[first], out[0]


def calibrate(x: np.ndarray, xs: np.ndarray, fit_values: np.ndarray) -> np.ndarray:
    """Scores read on a curve as the reference's `calibrate` does (README.md:53-56): the
    left search position clamped to [1, g - 1] (index -1 is the last point), t in the scores'
    dtype clamped to [0, 1] (NaN kept), then the lerp in float64."""
    g = xs.size
    i = np.searchsorted(xs, x, side="left")
    i = np.minimum(np.maximum(i, 1), g - 1)
    im1 = np.where(i == 0, g - 1, i - 1)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = (x - xs[im1]) / (xs[i] - xs[im1])
    t = np.where(t < 0, np.zeros_like(t), t)
    t = np.where(t > 1, np.ones_like(t), t)
    f0, f1 = fit_values[im1], fit_values[i]
    return f0 + t.astype(np.float64) * (f1 - f0)


def soft_rank(x: np.ndarray, strength: float, g: np.ndarray | None = None,
              precision: int = PREC_EXTENDED):
    """Soft ranks of the rows of x (the composition of the reference's paper/soft_rank.py:31-55:
    sort descending, non-increasing fit of s - (n..1), s - fit back in the input's order) with
    the oracle's fit; given an upstream g, also the gradient g - P^T A P g, scaled."""
    scale = 1.0 / strength
    x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]))
    n = x2.shape[1]
    theta = x2 * x2.dtype.type(scale)
    perm = np.argsort(-theta, axis=-1, kind="stable")
    s = np.take_along_axis(theta, perm, axis=-1)
    z = s - np.arange(n, 0, -1, dtype=x2.dtype)
    dual, starts = fit(z, None, increasing=False, precision=precision)
    out = np.empty_like(s)
    np.put_along_axis(out, perm, s - dual, axis=-1)
    if g is None:
        return out.reshape(x.shape), None
    g2 = np.ascontiguousarray(g.reshape(x2.shape).astype(x2.dtype))
    avg, _ = grad(dual, starts, np.take_along_axis(g2, perm, axis=-1))
    back = np.empty_like(avg)
    np.put_along_axis(back, perm, avg, axis=-1)
    return out.reshape(x.shape), ((g2 - back) * x2.dtype.type(scale)).reshape(x.shape)
