"""The CUDA operators, through the C ABI of include/tiso.h (libtiso.so, prebuilt for sm_100a).

Mirrors the reference's operator layer (src/torchisotonic/_ext.py:18-40): ``isotonic_tiles``
(the forward fit of [batch, n] rows and where its blocks start) and ``isotonic_grad`` (the
gradients from those block starts). Torch allocates every buffer, the workspace included, and
the kernels run on the current CUDA stream. There is no CPU implementation and no fallback:
without the library or a CUDA tensor these raise.
"""

from __future__ import annotations

import contextlib
import ctypes
import functools
import threading
from pathlib import Path

import torch
from torch import Tensor

LIB_PATH = Path(__file__).resolve().parent / "libtiso.so"

F16, BF16, F32, F64 = 0, 1, 2, 3
INCREASING, EXACT, CLIP_LO, CLIP_HI, WANT_GRAD_W = 1, 2, 4, 8, 16
ABI_VERSION = 2

_DTYPES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.float64: F64}


@functools.cache
def lib() -> ctypes.CDLL:
    """libtiso.so, loaded once. Raises if it was not built."""
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m torchisotonic_b200.build` "
            "(torchisotonic_b200 has no CPU fallback)"
        )
    so = ctypes.CDLL(str(LIB_PATH))
    p, i64, i32, u32, dbl, sz = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint,
                                 ctypes.c_double, ctypes.c_size_t)
    so.tiso_fit_workspace_size.argtypes = [i32, i32, i64, i64, u32, ctypes.POINTER(sz)]
    so.tiso_fit.argtypes = [i32, p, p, p, p, i64, i64, u32, dbl, dbl, p, p, sz, p]
    so.tiso_grad_workspace_size.argtypes = [i32, i32, i64, i64, u32, ctypes.POINTER(sz)]
    so.tiso_grad.argtypes = [i32, p, p, p, p, p, p, i64, i64, u32, dbl, dbl, p, sz, p]
    so.tiso_segment_blocks_workspace_size.argtypes = [i32, i32, i64, u32, ctypes.POINTER(sz)]
    so.tiso_segment_blocks.argtypes = [i32, p, p, i64, i64, u32, dbl, p, p, p, p, p, p, p, p, sz,
                                       p]
    so.tiso_segment_tile_count.argtypes = [i64, ctypes.POINTER(i64)]
    so.tiso_segment_expand_workspace_size.argtypes = [i32, ctypes.POINTER(sz)]
    so.tiso_segment_expand.argtypes = [i32, i32, i32, i64, p, p, p, p, p, i64, i64, u32, dbl,
                                       dbl, dbl, p, p, p, p, sz, p]
    so.tiso_segment_grad_workspace_size.argtypes = [i32, i32, i64, u32, ctypes.POINTER(sz)]
    so.tiso_segment_grad_sums.argtypes = [i32, p, p, p, p, i64, i64, u32, dbl, p, p, sz, p]
    so.tiso_segment_grad.argtypes = [i32, i32, i32, p, p, p, p, p, p, p, i64, i64, u32, dbl, dbl,
                                     dbl, p, sz, p]
    so.tiso_calib_groups_workspace_size.argtypes = [i32, i32, i64, i32, ctypes.POINTER(sz)]
    so.tiso_calib_groups.argtypes = [i32, p, i32, p, i64, i32, p, p, p, p, p, sz, p]
    so.tiso_calib_interp.argtypes = [i32, p, i64, p, p, i64, p, p]
    so.tiso_fit_varlen.argtypes = [i32, p, p, p, p, p, i64, i64, u32, dbl, dbl, p, p]
    so.tiso_check_weights.argtypes = [i32, p, i64, p, p]
    so.tiso_grad_varlen.argtypes = [i32, p, p, p, p, p, p, p, i64, i64, u32, dbl, dbl, p]
    so.tiso_last_error.restype = ctypes.c_char_p
    so.tiso_abi_version.restype = i32
    for f in ("tiso_fit_workspace_size", "tiso_fit", "tiso_grad_workspace_size", "tiso_grad",
              "tiso_segment_blocks_workspace_size", "tiso_segment_blocks", "tiso_segment_tile_count",
              "tiso_segment_expand_workspace_size", "tiso_segment_expand",
              "tiso_segment_grad_workspace_size", "tiso_segment_grad_sums", "tiso_segment_grad",
              "tiso_calib_groups_workspace_size", "tiso_calib_groups", "tiso_calib_interp",
              "tiso_fit_varlen", "tiso_grad_varlen", "tiso_check_weights"):
        getattr(so, f).restype = i32
    if so.tiso_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH} has ABI {so.tiso_abi_version()}, expected {ABI_VERSION}")
    return so


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(f"torchisotonic_b200: {lib().tiso_last_error().decode()} (status {rc})")


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


@functools.lru_cache(maxsize=256)
def _workspace_bytes(query_name: str, dtype: int, weighted: bool, batch: int, n: int,
                     flags: int) -> int:
    size = ctypes.c_size_t(0)
    _check(getattr(lib(), query_name)(dtype, int(weighted), batch, n, flags, ctypes.byref(size)))
    return size.value


def _workspace(query, dtype: int, weighted: bool, batch: int, n: int, flags: int,
               device: torch.device) -> tuple[Tensor | None, int]:
    name = getattr(query, "__name__", "")
    if name.startswith("tiso_"):  # a query of the library: its answer is cached
        size = _workspace_bytes(name, dtype, weighted, batch, n, flags)
    else:
        c_size = ctypes.c_size_t(0)
        _check(query(dtype, int(weighted), batch, n, flags, ctypes.byref(c_size)))
        size = c_size.value
    if size == 0:
        return None, 0
    # the caching allocator hands out 512-byte aligned blocks
    return torch.empty(size, dtype=torch.uint8, device=device), size


def _on(device: torch.device):
    """The device as the current one for the call (no switch when it is already)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _rows(y: Tensor, name: str) -> None:
    if not y.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: torchisotonic_b200 has no CPU path")
    if y.dim() != 2 or y.size(1) < 1 or not y.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous [batch, n] tensor with n >= 1")
    if y.dtype not in _DTYPES:
        raise RuntimeError(f"{name} must be float16, bfloat16, float32 or float64")


def acc_dtype(dtype: torch.dtype) -> torch.dtype:
    return torch.float64 if dtype == torch.float64 else torch.float32


def isotonic_tiles(
    y: Tensor,
    w: Tensor | None,
    increasing: bool,
    exact: bool = True,
    with_starts: bool = False,
    y_min: float | None = None,
    y_max: float | None = None,
    bad_weight: Tensor | None = None,
) -> tuple[Tensor, Tensor]:
    """The fit of every row of ``y`` ([batch, n], CUDA), clipped to [y_min, y_max] and in y's
    dtype, and if ``with_starts`` a bool tensor marking where its blocks start (else an empty
    one). ``w``: weights in the accumulation dtype (float64 for float64 data, else float32).
    ``bad_weight``: an int32 CUDA tensor of one element, set to 1 if a weight is not > 0."""
    _rows(y, "y")
    if w is not None:
        if w.shape != y.shape or w.dtype != acc_dtype(y.dtype) or not w.is_contiguous():
            raise RuntimeError("w must be contiguous, shaped like y, in y's accumulation dtype")
        if w.device != y.device:
            raise RuntimeError("w must be on y's device")
    batch, n = y.shape
    dtype = _DTYPES[y.dtype]
    flags = (INCREASING if increasing else 0) | (EXACT if exact else 0)
    flags |= (CLIP_LO if y_min is not None else 0) | (CLIP_HI if y_max is not None else 0)
    out = torch.empty_like(y)
    starts = (torch.empty(y.shape, dtype=torch.bool, device=y.device) if with_starts
              else torch.empty(0, dtype=torch.bool, device=y.device))
    so = lib()
    with _on(y.device):
        ws, ws_bytes = _workspace(so.tiso_fit_workspace_size, dtype, w is not None, batch, n,
                                  flags, y.device)
        stream = torch.cuda.current_stream(y.device).cuda_stream
        _check(so.tiso_fit(dtype, _ptr(y), _ptr(w), _ptr(out),
                           _ptr(starts) if with_starts else None, batch, n, flags,
                           0.0 if y_min is None else float(y_min),
                           0.0 if y_max is None else float(y_max),
                           _ptr(bad_weight), _ptr(ws), ws_bytes, stream))
    return out, starts


class WeightCheck:
    """The weights' check (any not > 0 fails; the reference synchronises on bool((w > 0).all())
    before its fit, src/torchisotonic/_api.py:60). For weights of up to EARLY_CHECK_BYTES, one
    pass of its own ahead of the fit (tiso_check_weights), its flag copied to pinned host memory
    behind an event: `failed()` waits for that pass alone while the fit launched after it runs,
    so the host's work around a short fit overlaps it. For larger weights the fit's own fused
    check (`flag`, to pass as the fit's bad_weight), read once the fit is done: a long fit hides
    the host's work anyway, and a second pass over the weights would cost more."""

    EARLY_CHECK_BYTES = 64 << 20

    class _Slot:
        """A device flag, a pinned host word and an event, reused by the calls of one thread on
        one device (allocating them took a noticeable part of a short call's host time)."""

        def __init__(self, dev: torch.device):
            self.flag = torch.empty(1, dtype=torch.int32, device=dev)
            self.host = torch.empty(1, dtype=torch.int32, pin_memory=True)
            self.event = torch.cuda.Event()
            self.busy = False

    _slots = threading.local()

    @classmethod
    def _take(cls, dev: torch.device) -> WeightCheck._Slot:
        slots = getattr(cls._slots, "by_device", None)
        if slots is None:
            slots = cls._slots.by_device = {}
        slot = slots.get(dev)
        if slot is None:
            slot = slots[dev] = cls._Slot(dev)
        elif slot.busy:  # left in use by a call that never read its flag: not reused
            slot = cls._Slot(dev)
        slot.busy = True
        return slot

    def __init__(self, w: Tensor):
        dev = w.device
        self._slot = self._take(dev)
        self.flag = self._slot.flag
        self.early = w.numel() * w.element_size() <= self.EARLY_CHECK_BYTES
        if not self.early:
            return
        with _on(dev):
            _check(lib().tiso_check_weights(_DTYPES[w.dtype], _ptr(w), w.numel(), _ptr(self.flag),
                                            torch.cuda.current_stream(dev).cuda_stream))
            self._slot.host.copy_(self.flag, non_blocking=True)
            self._slot.event.record()

    @property
    def fused_flag(self) -> Tensor | None:
        """The flag the fit itself should set (None when the early pass checks the weights)."""
        return None if self.early else self.flag

    def failed(self) -> bool:
        if self.early:
            self._slot.event.synchronize()
            bad = bool(self._slot.host.item())
        else:
            bad = bool(self.flag.item())
        self._slot.busy = False
        return bad


def isotonic_grad(
    starts: Tensor,
    g: Tensor,
    w: Tensor | None,
    y: Tensor | None,
    want_y: bool = True,
    want_w: bool = False,
    y_min: float | None = None,
    y_max: float | None = None,
) -> tuple[Tensor | None, Tensor | None]:
    """Gradients of sum(fit * g) in y (y's dtype) and, with ``want_w``, in w (accumulation
    dtype), from the fit's block ``starts``. ``y`` is needed for ``want_w`` or a clipped fit:
    the kernel recomputes the fit (each block's mean) from it. Mirrors the reference's
    isotonic_grad (src/torchisotonic/_ext.py:34-40)."""
    _rows(g, "g")
    if starts.shape != g.shape or starts.dtype != torch.bool or not starts.is_contiguous():
        raise RuntimeError("starts must be a contiguous bool tensor shaped like g")
    if y is not None and (y.shape != g.shape or y.dtype != g.dtype or not y.is_contiguous()):
        raise RuntimeError("y must be contiguous and shaped and typed like g")
    if w is not None and (w.shape != g.shape or w.dtype != acc_dtype(g.dtype)
                          or not w.is_contiguous()):
        raise RuntimeError("w must be contiguous, shaped like g, in the accumulation dtype")
    batch, n = g.shape
    dtype = _DTYPES[g.dtype]
    flags = (CLIP_LO if y_min is not None else 0) | (CLIP_HI if y_max is not None else 0)
    flags |= WANT_GRAD_W if want_w else 0
    gy = torch.empty_like(g) if want_y else None
    gw = torch.empty(g.shape, dtype=acc_dtype(g.dtype), device=g.device) if want_w else None
    so = lib()
    with _on(g.device):
        ws, ws_bytes = _workspace(so.tiso_grad_workspace_size, dtype, w is not None, batch, n,
                                  flags, g.device)
        stream = torch.cuda.current_stream(g.device).cuda_stream
        _check(so.tiso_grad(dtype, _ptr(y), _ptr(w), _ptr(starts), _ptr(g), _ptr(gy), _ptr(gw),
                            batch, n, flags, 0.0 if y_min is None else float(y_min),
                            0.0 if y_max is None else float(y_max), _ptr(ws), ws_bytes, stream))
    return gy, gw


def row_offset(first: float) -> float:
    """The offset y0 of a row from its first element (the kernels' rule, csrc/common.cuh
    offset_of): v cut to 8 significant bits if |v| >= 1 (and finite), else 0."""
    import math
    import struct

    if not (abs(first) >= 1.0) or math.isinf(first):
        return 0.0
    bits = struct.unpack("<q", struct.pack("<d", first))[0]
    bits &= ~((1 << 45) - 1)
    return struct.unpack("<d", struct.pack("<q", bits))[0]


def segment_blocks(y: Tensor, w: Tensor | None, seg_start: int, increasing: bool, y0: float,
                   bad_weight: Tensor | None = None):
    """The fitted blocks of one segment (1-D CUDA tensors y, w) of a row split across devices:
    (lists, count int32[1], nan int32[1], tile_offs int64[tiles + 1]). lists is one [3, n] int64
    tensor: row 0 each block's first element, rows 1 and 2 its T and W (float64 bits; `.view(
    torch.float64)`), capacity n; tile_offs where each 512-element tile's blocks begin."""
    if not y.is_cuda or y.dim() != 1 or not y.is_contiguous() or y.dtype not in _DTYPES:
        raise RuntimeError("y must be a contiguous 1-D float CUDA tensor")
    if w is not None and (w.shape != y.shape or w.dtype != acc_dtype(y.dtype)
                          or not w.is_contiguous()):
        raise RuntimeError("w must be contiguous, shaped like y, in y's accumulation dtype")
    n = y.numel()
    dev = y.device
    flags = (INCREASING if increasing else 0) | EXACT
    lists = torch.empty(3, n, dtype=torch.int64, device=dev)
    count = torch.zeros(1, dtype=torch.int32, device=dev)
    nan = torch.zeros(1, dtype=torch.int32, device=dev)
    so = lib()
    tiles = ctypes.c_int64()
    _check(so.tiso_segment_tile_count(n, ctypes.byref(tiles)))
    tile_offs = torch.empty(tiles.value + 1, dtype=torch.int64, device=dev)
    with _on(dev):
        ws, ws_bytes = _workspace(lambda d, wt, b, nn, f, r: so.tiso_segment_blocks_workspace_size(
            d, wt, nn, f, r), _DTYPES[y.dtype], w is not None, 1, n, flags, dev)
        _check(so.tiso_segment_blocks(_DTYPES[y.dtype], _ptr(y), _ptr(w), n, seg_start, flags,
                                      float(y0), _ptr(lists[0]), _ptr(lists[1]), _ptr(lists[2]),
                                      _ptr(count), _ptr(nan), _ptr(bad_weight), _ptr(tile_offs),
                                      _ptr(ws), ws_bytes,
                                      torch.cuda.current_stream(dev).cuda_stream))
    return lists, count, nan, tile_offs


def segment_expand(dtype: torch.dtype, parts: int, me: int, cap: int, starts: Tensor, t: Tensor,
                   wsum: Tensor, counts: Tensor, nans: Tensor, seg_n: int, seg_start: int,
                   increasing: bool, y0: float, y_min: float | None, y_max: float | None,
                   with_starts: bool = False, tile_offs: Tensor | None = None):
    """The fit of segment `me` from the gathered block lists of all `parts` segments (list k at
    offset k * cap; t and wsum are merged in place). tile_offs: this segment's tile offsets from
    segment_blocks (each tile's blocks found directly), or None (searched in the whole list)."""
    dev = t.device
    flags = (INCREASING if increasing else 0) | EXACT
    flags |= (CLIP_LO if y_min is not None else 0) | (CLIP_HI if y_max is not None else 0)
    out = torch.empty(seg_n, dtype=dtype, device=dev)
    st = torch.empty(seg_n, dtype=torch.bool, device=dev) if with_starts else None
    so = lib()
    with _on(dev):
        size = ctypes.c_size_t()
        _check(so.tiso_segment_expand_workspace_size(parts, ctypes.byref(size)))
        ws = torch.empty(size.value, dtype=torch.uint8, device=dev)
        _check(so.tiso_segment_expand(_DTYPES[dtype], parts, me, cap, _ptr(starts), _ptr(t),
                                      _ptr(wsum), _ptr(counts), _ptr(nans), seg_n, seg_start,
                                      flags, float(y0), 0.0 if y_min is None else float(y_min),
                                      0.0 if y_max is None else float(y_max), _ptr(out), _ptr(st),
                                      _ptr(tile_offs), _ptr(ws), size.value,
                                      torch.cuda.current_stream(dev).cuda_stream))
    return out, st


def _grad_flags(want_w: bool, y_min: float | None, y_max: float | None) -> int:
    return ((WANT_GRAD_W if want_w else 0) | (CLIP_LO if y_min is not None else 0)
            | (CLIP_HI if y_max is not None else 0))


def segment_grad_workspace(dtype: torch.dtype, weighted: bool, seg_n: int, device) -> Tensor:
    size = ctypes.c_size_t()
    _check(lib().tiso_segment_grad_workspace_size(_DTYPES[dtype], int(weighted), seg_n, 0,
                                                  ctypes.byref(size)))
    return torch.empty(size.value, dtype=torch.uint8, device=device)


def segment_grad_sums(y: Tensor, w: Tensor | None, starts: Tensor, g: Tensor, seg_start: int,
                      y0: float, want_w: bool, y_min: float | None, y_max: float | None,
                      ws: Tensor) -> Tensor:
    """Step 1 of a split row's backward: the segment's run, 10 float64 (device)."""
    run = torch.empty(10, dtype=torch.float64, device=g.device)
    flags = _grad_flags(want_w, y_min, y_max)
    with torch.cuda.device(g.device):
        _check(lib().tiso_segment_grad_sums(
            _DTYPES[g.dtype], _ptr(y), _ptr(w), _ptr(starts), _ptr(g), g.numel(), seg_start,
            flags, float(y0), _ptr(run), _ptr(ws), ws.numel(),
            torch.cuda.current_stream(g.device).cuda_stream))
    return run


def segment_grad(parts: int, me: int, runs: Tensor, y: Tensor | None, w: Tensor | None,
                 starts: Tensor, g: Tensor, seg_start: int, y0: float, want_w: bool,
                 y_min: float | None, y_max: float | None, ws: Tensor):
    """Step 2: (grad_y, grad_w or None) of segment `me` from the gathered runs [parts, 10]."""
    gy = torch.empty_like(g)
    gw = torch.empty(g.shape, dtype=acc_dtype(g.dtype), device=g.device) if want_w else None
    flags = _grad_flags(want_w, y_min, y_max)
    with torch.cuda.device(g.device):
        _check(lib().tiso_segment_grad(
            _DTYPES[g.dtype], parts, me, _ptr(runs), _ptr(y), _ptr(w), _ptr(starts), _ptr(g),
            _ptr(gy), _ptr(gw), g.numel(), seg_start, flags, float(y0),
            0.0 if y_min is None else float(y_min), 0.0 if y_max is None else float(y_max),
            _ptr(ws), ws.numel(), torch.cuda.current_stream(g.device).cuda_stream))
    return gy, gw


def calib_groups(scores: Tensor, labels: Tensor,
                 presorted: bool = False) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """The pre-step of a calibration curve: the n (score, label) pairs (1-D contiguous CUDA
    tensors; scores float32/float64, labels float32/float64) sorted by score (``presorted``:
    they come sorted), equal scores pooled. Returns (xs, y, w, groups): per distinct score, in increasing order, the score
    (scores' dtype), the mean label and the count (float64), each of capacity n, and groups, an
    int64[2] CUDA tensor holding their number G and a NaN-score flag."""
    n = scores.numel()
    dev = scores.device
    xs = torch.empty(n, dtype=scores.dtype, device=dev)
    y = torch.empty(n, dtype=torch.float64, device=dev)
    w = torch.empty(n, dtype=torch.float64, device=dev)
    groups = torch.empty(2, dtype=torch.int64, device=dev)
    kd, ld = _DTYPES[scores.dtype], _DTYPES[labels.dtype]
    so = lib()
    with torch.cuda.device(dev):
        size = ctypes.c_size_t()
        _check(so.tiso_calib_groups_workspace_size(kd, ld, n, int(presorted), ctypes.byref(size)))
        ws = torch.empty(size.value, dtype=torch.uint8, device=dev)
        _check(so.tiso_calib_groups(kd, _ptr(scores), ld, _ptr(labels), n, int(presorted),
                                    _ptr(xs), _ptr(y),
                                    _ptr(w), _ptr(groups), _ptr(ws), size.value,
                                    torch.cuda.current_stream(dev).cuda_stream))
    return xs, y, w, groups


def calib_interp(x: Tensor, xs: Tensor, fit: Tensor) -> Tensor:
    """The scores x (1-D contiguous CUDA, xs's dtype) read on the curve (xs, fit float64):
    float64, linear between its points and constant beyond them."""
    out = torch.empty(x.numel(), dtype=torch.float64, device=x.device)
    with torch.cuda.device(x.device):
        _check(lib().tiso_calib_interp(_DTYPES[x.dtype], _ptr(x), x.numel(), _ptr(xs), _ptr(fit),
                                       xs.numel(), _ptr(out),
                                       torch.cuda.current_stream(x.device).cuda_stream))
    return out


# ---------------------------------------------------------------------------------------------
# Ragged rows: packed back to back, row r = [offsets[r], offsets[r + 1])

VARLEN_MAX = 512


def _varlen_args(y: Tensor, offsets: Tensor, max_len: int) -> int:
    if not y.is_cuda:
        raise RuntimeError("y must be a CUDA tensor: torchisotonic_b200 has no CPU path")
    if y.dim() != 1 or not y.is_contiguous() or y.dtype not in _DTYPES:
        raise RuntimeError("y must be a contiguous 1-D float16, bfloat16, float32 or float64 tensor")
    if (offsets.dim() != 1 or offsets.dtype != torch.int64 or not offsets.is_contiguous()
            or offsets.device != y.device or offsets.numel() < 1):
        raise RuntimeError("offsets must be a contiguous 1-D int64 tensor on y's device")
    if not 0 <= max_len <= VARLEN_MAX:
        raise RuntimeError(f"ragged rows must have at most {VARLEN_MAX} elements")
    return offsets.numel() - 1


def isotonic_tiles_varlen(
    y: Tensor,
    w: Tensor | None,
    offsets: Tensor,
    max_len: int,
    increasing: bool,
    exact: bool = True,
    with_starts: bool = False,
    y_min: float | None = None,
    y_max: float | None = None,
    bad_weight: Tensor | None = None,
) -> tuple[Tensor, Tensor]:
    """The fit of every ragged row of the packed ``y`` (1-D, CUDA; row r is
    y[offsets[r]:offsets[r + 1]], each at most ``max_len`` long), clipped and in y's dtype, and
    if ``with_starts`` where its blocks start (else an empty tensor)."""
    batch = _varlen_args(y, offsets, max_len)
    if w is not None and (w.shape != y.shape or w.dtype != acc_dtype(y.dtype)
                          or not w.is_contiguous() or w.device != y.device):
        raise RuntimeError("w must be contiguous, shaped like y, in y's accumulation dtype")
    flags = (INCREASING if increasing else 0) | (EXACT if exact else 0)
    flags |= (CLIP_LO if y_min is not None else 0) | (CLIP_HI if y_max is not None else 0)
    out = torch.empty_like(y)
    starts = (torch.empty(y.shape, dtype=torch.bool, device=y.device) if with_starts
              else torch.empty(0, dtype=torch.bool, device=y.device))
    with torch.cuda.device(y.device):
        _check(lib().tiso_fit_varlen(_DTYPES[y.dtype], _ptr(y), _ptr(w), _ptr(out),
                                     _ptr(starts) if with_starts else None, _ptr(offsets), batch,
                                     max_len, flags, 0.0 if y_min is None else float(y_min),
                                     0.0 if y_max is None else float(y_max), _ptr(bad_weight),
                                     torch.cuda.current_stream(y.device).cuda_stream))
    return out, starts


def isotonic_grad_varlen(
    starts: Tensor,
    g: Tensor,
    w: Tensor | None,
    y: Tensor | None,
    offsets: Tensor,
    max_len: int,
    want_y: bool = True,
    want_w: bool = False,
    y_min: float | None = None,
    y_max: float | None = None,
) -> tuple[Tensor | None, Tensor | None]:
    """isotonic_grad over ragged rows (packed 1-D tensors, row r = [offsets[r], offsets[r + 1]))."""
    batch = _varlen_args(g, offsets, max_len)
    if starts.shape != g.shape or starts.dtype != torch.bool or not starts.is_contiguous():
        raise RuntimeError("starts must be a contiguous bool tensor shaped like g")
    if y is not None and (y.shape != g.shape or y.dtype != g.dtype or not y.is_contiguous()):
        raise RuntimeError("y must be contiguous and shaped and typed like g")
    if w is not None and (w.shape != g.shape or w.dtype != acc_dtype(g.dtype)
                          or not w.is_contiguous()):
        raise RuntimeError("w must be contiguous, shaped like g, in the accumulation dtype")
    flags = (CLIP_LO if y_min is not None else 0) | (CLIP_HI if y_max is not None else 0)
    flags |= WANT_GRAD_W if want_w else 0
    gy = torch.empty_like(g) if want_y else None
    gw = torch.empty(g.shape, dtype=acc_dtype(g.dtype), device=g.device) if want_w else None
    with torch.cuda.device(g.device):
        _check(lib().tiso_grad_varlen(_DTYPES[g.dtype], _ptr(y), _ptr(w), _ptr(starts), _ptr(g),
                                      _ptr(gy), _ptr(gw), _ptr(offsets), batch, max_len, flags,
                                      0.0 if y_min is None else float(y_min),
                                      0.0 if y_max is None else float(y_max),
                                      torch.cuda.current_stream(g.device).cuda_stream))
    return gy, gw
