"""tiso_grad_noalloc, the backward entry point that allocates nothing.

Some callers cannot allocate device memory when they call the library: a host that links only
this library and the CUDA runtime and has no device allocator of its own to hand (a plain C or
foreign-language caller), or one whose device memory is budgeted up front. For them
tiso_grad_noalloc takes no workspace; long rows use a fixed scratch array inside the library.
These tests call it through the C ABI and compare it with the oracle's gradients and with
tiso_grad (given a workspace), on two calls in a row - the second with other data, since every
call reuses the same scratch - including rows of more than 1024 tiles, whose row scan runs in
chunks and keeps its chunk totals in the same scratch. This file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from torchisotonic_b200 import _ext


def _noalloc():
    so = _ext.lib()
    p, i64, i32, u32, dbl = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint,
                             ctypes.c_double)
    f = so.tiso_grad_noalloc
    f.argtypes = [i32, p, p, p, p, p, p, i64, i64, u32, dbl, dbl, p]
    f.restype = i32
    return so, f


def _case(seed: int, batch: int, n: int, dtype: torch.dtype, weighted: bool):
    """Inputs on the GPU, and the oracle's block starts (of its own fit) and gradients."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    acc = _ext.acc_dtype(dtype)
    y = (torch.linspace(0, 3, n, device="cuda", dtype=torch.float64)
         + torch.randn(batch, n, generator=g, device="cuda", dtype=torch.float64)).to(dtype)
    w = (torch.rand(batch, n, generator=g, device="cuda", dtype=acc) + 0.1) if weighted else None
    c = torch.randn(batch, n, generator=g, device="cuda", dtype=torch.float64).to(dtype)
    yn = y.to(acc).cpu().numpy()
    wn = None if w is None else w.cpu().numpy()
    fit, st = oracle.fit(yn, wn)
    oy, ow = oracle.grad(fit, st, c.to(acc).cpu().numpy(), wn, yn, y_min=0.5, y_max=2.5)
    starts = torch.from_numpy(st).cuda()
    return y, w, c, starts, oy, ow


def _call_noalloc(f, y, w, c, starts, flags, lo, hi):
    gy = torch.empty_like(c)
    gw = torch.empty(c.shape, dtype=_ext.acc_dtype(c.dtype), device="cuda")
    want_w = bool(flags & _ext.WANT_GRAD_W)
    rc = f(_ext._DTYPES[c.dtype], y.data_ptr(), None if w is None else w.data_ptr(),
           starts.data_ptr(), c.data_ptr(), gy.data_ptr(), gw.data_ptr() if want_w else None,
           c.shape[0], c.shape[1], flags, lo, hi,
           torch.cuda.current_stream().cuda_stream)
    return rc, gy, gw


@pytest.mark.gpu
@pytest.mark.parametrize(
    ("dtype", "weighted", "batch", "n"),
    [(torch.float64, True, 6, 5000),       # long rows: five 1024-tiles each, fixed scratch
     (torch.float32, False, 4, 70_000),    # 69 tiles per row
     (torch.float32, False, 2, 1_100_000), # 1075 tiles per row: the row scan runs in chunks
     (torch.bfloat16, True, 3, 9000),
     (torch.float64, True, 50, 300)],      # short rows: no scratch at all
)
def test_noalloc_matches_the_oracle_and_the_workspace_entry_point(dtype, weighted, batch,
                                                                  n) -> None:
    so, f = _noalloc()
    flags = _ext.CLIP_LO | _ext.CLIP_HI | (_ext.WANT_GRAD_W if weighted else 0)
    lo, hi = 0.5, 2.5
    for seed in (1, 2):  # two calls in a row, on different data
        y, w, c, starts, oy, ow = _case(seed, batch, n, dtype, weighted)
        rc, gy, gw = _call_noalloc(f, y, w, c, starts, flags, lo, hi)
        assert rc == 0, so.tiso_last_error().decode()
        torch.cuda.synchronize()
        # against the oracle (independent of this library)
        if dtype == torch.bfloat16:
            rtol, atol = 2.0**-8, 2.0**-8
        else:
            rtol = atol = 1e-9 if dtype == torch.float64 else 2e-5
        np.testing.assert_allclose(gy.double().cpu().numpy(), oy.astype(np.float64),
                                   rtol=rtol, atol=atol)
        if weighted:
            np.testing.assert_allclose(gw.double().cpu().numpy(), ow.astype(np.float64),
                                       rtol=rtol, atol=atol * 4)
        # and against tiso_grad with a workspace (the same kernels: the same numbers)
        want_y, want_w = _ext.isotonic_grad(starts, c, w, y, True, weighted, lo, hi)
        assert torch.equal(gy, want_y)
        if weighted:
            assert torch.equal(gw, want_w)


@pytest.mark.gpu
def test_noalloc_refuses_problems_beyond_its_scratch() -> None:
    so, f = _noalloc()
    # 20 rows of 4,000,000 elements: 20 * 3907 tiles of 1024 > 32768. Refused before any launch,
    # so the (unused) pointers below are never dereferenced.
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    rc = f(_ext.F32, dummy.data_ptr(), None, dummy.data_ptr(), dummy.data_ptr(),
           dummy.data_ptr(), None, 20, 4_000_000, 0, 0.0, 0.0, None)
    assert rc == 2
    assert "32768" in so.tiso_last_error().decode()
