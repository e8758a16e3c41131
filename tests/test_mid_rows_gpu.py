"""Rows of 33..64 elements (the tile kernel's whole rows of up to 8 threads) and the backward of
rows of at most 64 elements (grad_rows_kernel: 8 elements a lane, 1 to 8 lanes a row) against
the oracle.

Every row length of the range's edges and some between, each dtype, weighted or not, both
directions, with clip and the block starts; patterns that make every element its own block,
one block, exact ties and NaN; rows whose byte length or start is not a multiple of 16 (the
element-wise loads and stores); non-positive weights through the C ABI.
"""

from __future__ import annotations

import math

import pytest
import torch

import oracle
from parity import check_fit, check_starts
from torchisotonic_b200 import _ext

pytestmark = pytest.mark.gpu

LENGTHS = [33, 34, 40, 47, 48, 56, 63, 64]


def _rows(n: int, batch: int, seed: int, kind: str = "trend") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    i = torch.arange(n, dtype=torch.float64)
    if kind == "trend":
        return torch.linspace(0, 3, n, dtype=torch.float64) + torch.randn(
            batch, n, generator=g, dtype=torch.float64)
    if kind == "increasing":
        return (i + 0.25 * torch.rand(batch, n, generator=g, dtype=torch.float64)).cumsum(1)
    if kind == "decreasing":
        return -i.expand(batch, n).clone()
    if kind == "ties":
        return torch.randint(0, 4, (batch, n), generator=g).double()
    if kind == "saw":
        return (i % 5 + 0.3 * i).expand(batch, n).clone()
    raise ValueError(kind)


@pytest.mark.parametrize("n", LENGTHS)
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.float16, torch.bfloat16])
def test_lengths_and_dtypes(n: int, dtype: torch.dtype) -> None:
    y = _rows(n, 300, n).to(dtype)
    w = 0.1 + torch.rand(300, n, generator=torch.Generator().manual_seed(n + 1))
    w = w.to(_ext.acc_dtype(dtype))
    check_fit(y)
    check_fit(y, increasing=False)
    check_fit(y, w)
    check_fit(y, w, increasing=False, y_min=-0.5, y_max=2.0)


@pytest.mark.parametrize("kind", ["increasing", "decreasing", "ties", "saw"])
@pytest.mark.parametrize("n", [33, 63, 64])
def test_patterns(kind: str, n: int) -> None:
    y = _rows(n, 70, 5 * n, kind)
    w = (0.1 + torch.rand(70, n, generator=torch.Generator().manual_seed(n))).double()
    for inc in (True, False):
        check_fit(y, increasing=inc)
        check_fit(y, w, increasing=inc)
        check_fit(y.float(), increasing=inc)
        check_fit(y.float(), w.float(), increasing=inc)


@pytest.mark.parametrize("n", [33, 64])
def test_float32_not_exact(n: int) -> None:
    y = _rows(n, 500, n).float()
    w = 0.1 + torch.rand(500, n, generator=torch.Generator().manual_seed(2))
    check_fit(y, exact=False)
    check_fit(y, w, exact=False, increasing=False)


def test_nan_rows() -> None:
    y = _rows(50, 40, 3)
    y[0, 0] = math.nan
    y[7, 33] = math.nan
    y[39, 49] = math.nan
    y[12, 10] = math.inf  # a lone infinity is a value, not NaN
    for t in (y, y.float()):
        check_fit(t, starts=False)
        _, st = _ext.isotonic_tiles(t.cuda(), None, True, True, True)
        st = st.cpu()
        for r in (0, 7, 39):
            assert st[r].tolist() == [True] + [False] * 49


@pytest.mark.parametrize("n", [33, 37, 64])
def test_unaligned_rows(n: int) -> None:
    # rows that start off a 16-byte boundary (a column slice, made contiguous by the API, and a
    # storage offset kept by the C ABI path): element-wise loads and stores
    big = _rows(n + 1, 130, n)
    y = big[:, 1:]
    check_fit(y)
    check_fit(y.float())
    flat = big.float().cuda().reshape(-1)[1:1 + 130 * n].reshape(130, n)
    assert flat.is_contiguous() and flat.data_ptr() % 16 != 0
    out, st = _ext.isotonic_tiles(flat, None, True, True, True)
    want, wst = oracle.fit(flat.cpu().double().numpy(), None, increasing=True)
    torch.testing.assert_close(out.cpu().double(), torch.from_numpy(want), rtol=2.4e-7,
                               atol=1e-6)
    assert (st.cpu().numpy() == wst).all()


def test_batch_edges() -> None:
    for batch in (1, 31, 32, 33, 65, 4097):
        y = _rows(48, batch, batch)
        check_fit(y)
        check_starts(y.float(), None, increasing=False)


def test_negative_weight_sets_the_flag_without_fault() -> None:
    # a weight that is not > 0 reaches the kernels through the C ABI: the flag is set and the
    # launch ends normally (no stack pools below its sentinel)
    for n in (20, 40, 64, 300):
        for dtype in (torch.float64, torch.float32):
            y = torch.zeros(64, n, dtype=dtype, device="cuda")
            w = -torch.ones(64, n, dtype=dtype, device="cuda")
            flag = torch.zeros(1, dtype=torch.int32, device="cuda")
            _ext.isotonic_tiles(y, w, True, True, True, bad_weight=flag)
            torch.cuda.synchronize()
            assert int(flag.item()) == 1


# ---- the backward of rows of at most 64 elements ----


def _grads(y, w, c, **kw):
    from test_grad_gpu import grads_cuda, grads_oracle
    gy, gw = grads_cuda(y, w, c, **kw)
    kw.pop("dim", None)
    oy, ow = grads_oracle(y, w, c, **kw)
    return gy, gw, oy, ow


GRAD_TOL = {torch.float64: 1e-9, torch.float32: 2e-5, torch.float16: 2.0**-10,
            torch.bfloat16: 2.0**-7}


@pytest.mark.parametrize("n", [1, 2, 5, 16, 17, 31, 48, 63, 64])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.float16, torch.bfloat16])
def test_short_row_gradients(n: int, dtype: torch.dtype) -> None:
    g = torch.Generator().manual_seed(7 * n)
    y = _rows(n, 90, n) if n >= 2 else torch.randn(90, 1, generator=g, dtype=torch.float64)
    y = y.to(dtype)
    w = (0.1 + torch.rand(90, n, generator=g)).to(_ext.acc_dtype(dtype))
    c = torch.randn(90, n, generator=g).to(dtype)
    tol = GRAD_TOL[dtype]
    for kw in ({}, {"increasing": False}, {"y_min": 0.5, "y_max": 2.5}):
        for ww in (None, w):
            gy, gw, oy, ow = _grads(y, ww, c, **kw)
            torch.testing.assert_close(gy.double(), oy.to(dtype).double(), rtol=tol, atol=tol,
                                       equal_nan=True)
            if ww is not None:
                scale = 1 + float(y.double().abs().max())
                torch.testing.assert_close(gw.double(), ow.double(), rtol=max(tol, 1e-6),
                                           atol=max(tol, 1e-6) * scale, equal_nan=True)


@pytest.mark.parametrize("n", [17, 37, 64])
def test_gradients_one_side_and_unaligned(n: int) -> None:
    # only d/dw or only d/dy wanted, and rows whose start is off a 16-byte boundary (storage
    # offsets through the C ABI)
    g = torch.Generator().manual_seed(n)
    big = _rows(n, 130, n).float().cuda().reshape(-1)
    y = big[1:1 + 129 * n].reshape(129, n)
    wb = (0.1 + torch.rand(130 * n, generator=g)).cuda()
    w = wb[3:3 + 129 * n].reshape(129, n)
    cb = torch.randn(130 * n, generator=g).cuda()
    c = cb[1:1 + 129 * n].reshape(129, n)
    assert y.data_ptr() % 16 and w.data_ptr() % 16 and c.data_ptr() % 16
    out, st = _ext.isotonic_tiles(y, w, True, True, True)
    gy_both, gw_both = _ext.isotonic_grad(st, c, w, y, True, True)
    gy_only, none_w = _ext.isotonic_grad(st, c, w, y, True, False)
    none_y, gw_only = _ext.isotonic_grad(st, c, w, y, False, True)
    assert none_w is None and none_y is None
    assert torch.equal(gy_both, gy_only) and torch.equal(gw_both, gw_only)
    fy, fw = y.cpu().double().numpy(), w.cpu().double().numpy()
    fit, wst = oracle.fit(fy, fw, increasing=True)
    assert (st.cpu().numpy() == wst).all()
    oy, ow = oracle.grad(fit, wst, c.cpu().double().numpy(), fw, fy)
    torch.testing.assert_close(gy_both.cpu().double(), torch.from_numpy(oy), rtol=2e-5,
                               atol=2e-5)
    torch.testing.assert_close(gw_both.cpu().double(), torch.from_numpy(ow), rtol=2e-5,
                               atol=2e-5 * (1 + float(y.abs().max())))
