"""Ragged rows on the GPU (torchisotonic_b200.isotonic_varlen, tiso_fit_varlen / tiso_grad_varlen):
every row fitted at its own length, against the oracle fitting each row alone; the padded batch
that the reference's README describes for rows of unequal length (README.md:100-103) against the
packed rows; gradients; the C ABI called directly."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch
from parity import assert_values, scale_of

import oracle
import torchisotonic_b200
from torchisotonic_b200 import _ext

pytestmark = pytest.mark.gpu


def _offsets(lengths: list[int], base: int = 0) -> torch.Tensor:
    return torch.tensor([base] + list(np.cumsum(lengths) + base), dtype=torch.int64)


def _oracle_rows(values: torch.Tensor, offsets: torch.Tensor, w: torch.Tensor | None, **kw):
    """The oracle's fit and block starts of every row alone (rows of one length fitted together)."""
    off = offsets.tolist()
    out = torch.empty_like(values)
    starts = torch.zeros(values.shape, dtype=torch.bool)
    lens = [off[r + 1] - off[r] for r in range(len(off) - 1)]
    for length in sorted(set(lens)):
        rows = [r for r, n in enumerate(lens) if n == length]
        if length == 0:
            continue
        idx = torch.tensor([list(range(off[r], off[r] + length)) for r in rows])
        y2 = values[idx]
        w2 = None if w is None else w[idx]
        res, st = oracle.isotonic(y2, w2, with_starts=True, **kw)
        out[idx] = res
        starts[idx] = st.reshape(y2.shape)
    return out, starts


def _check(values, offsets, w=None, exact=True, max_len=None, **kw):
    got = torchisotonic_b200.isotonic_varlen(
        values.cuda(), offsets.cuda(), None if w is None else w.cuda(), exact=exact,
        max_len=max_len, **kw)
    want, wst = _oracle_rows(values, offsets, w, **kw)
    base = int(offsets[0])
    end = int(offsets[-1])
    assert got.shape == values.shape and got.dtype == want.dtype
    assert_values(got[base:end], want[base:end], scale_of(values), exact=exact)
    if exact or values.dtype == torch.float64:
        acc = torch.float64 if values.dtype == torch.float64 else torch.float32
        _, st = _ext.isotonic_tiles_varlen(
            values.cuda(), None if w is None else w.cuda().to(acc), offsets.cuda(),
            int(max_len if max_len is not None else (offsets[1:] - offsets[:-1]).max()),
            kw.get("increasing", True), True, True)
        assert torch.equal(st.cpu()[base:end], wst[base:end])


def _ragged(lengths, g, dtype=torch.float32, weighted=False, base=0):
    total = base + sum(lengths)
    y = torch.zeros(total, dtype=torch.float64)
    off = _offsets(lengths, base)
    for r, n in enumerate(lengths):
        s0 = int(off[r])
        y[s0:s0 + n] = torch.linspace(0, 2, n, dtype=torch.float64) + torch.randn(n, generator=g,
                                                                               dtype=torch.float64)
    w = None
    if weighted:
        w = (torch.rand(total, generator=g, dtype=torch.float64) + 0.1)
        w = w.to(torch.float64 if dtype == torch.float64 else torch.float32)
    return y.to(dtype), off, w


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize("increasing", [True, False])
def test_random_lengths(dtype, weighted, increasing) -> None:
    g = torch.Generator().manual_seed(11)
    lengths = torch.randint(0, 513, (300,), generator=g).tolist()
    y, off, w = _ragged(lengths, g, dtype, weighted)
    _check(y, off, w, increasing=increasing)


@pytest.mark.parametrize("n", [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256,
                               257, 511, 512])
def test_one_length_equals_the_padded_kernels(n: int) -> None:
    # rows all of length n: the same fit (bit for bit) and starts as isotonic() on [batch, n]
    g = torch.Generator().manual_seed(n)
    y = (torch.linspace(0, 3, n) + torch.randn(97, n, generator=g)).cuda()
    w = (torch.rand(97, n, generator=g) + 0.1).cuda()
    off = (torch.arange(98, dtype=torch.int64) * n).cuda()
    for ww in (None, w):
        fixed = torchisotonic_b200.isotonic(y, ww, y_min=0.1, y_max=2.5)
        var = torchisotonic_b200.isotonic_varlen(y.reshape(-1), off, None if ww is None else
                                                 ww.reshape(-1), y_min=0.1, y_max=2.5)
        assert torch.equal(var.reshape(97, n), fixed)
        _, st_f = _ext.isotonic_tiles(y, ww, True, True, True)
        _, st_v = _ext.isotonic_tiles_varlen(y.reshape(-1), None if ww is None else ww.reshape(-1),
                                             off, n, True, True, True)
        assert torch.equal(st_v.reshape(97, n), st_f)


def test_clip_exact_false_nan_and_empty_rows() -> None:
    g = torch.Generator().manual_seed(5)
    lengths = [0, 1, 7, 0, 64, 300, 512, 0, 3, 33]
    y, off, w = _ragged(lengths, g, torch.float32, weighted=True)
    y[int(off[5]) + 17] = math.nan  # row 5 holds a NaN: all NaN, one block
    _check(y, off, w, y_min=0.2, y_max=1.8)
    _check(y, off, None, increasing=False, y_min=0.0)
    _check(y, off, w, exact=False)
    out = torchisotonic_b200.isotonic_varlen(y.cuda(), off.cuda(), w.cuda()).cpu()
    r5 = out[int(off[5]):int(off[6])]
    assert torch.isnan(r5).all()


def test_offsets_with_a_base_and_a_larger_max_len() -> None:
    g = torch.Generator().manual_seed(3)
    lengths = torch.randint(1, 200, (50,), generator=g).tolist()
    y, off, w = _ragged(lengths, g, torch.float64, weighted=True, base=37)
    _check(y, off, w, max_len=512)
    _check(y, off, w, max_len=max(lengths))


def test_rows_longer_than_max_len_are_cut() -> None:
    # a row longer than max_len: its first max_len elements are fitted as a row, the rest untouched
    g = torch.Generator().manual_seed(9)
    y = torch.randn(40, generator=g).cuda()
    off = torch.tensor([0, 10, 40], dtype=torch.int64).cuda()
    out = torch.full((40,), 123.0, device="cuda")
    flags = _ext.INCREASING | _ext.EXACT
    rc = _ext.lib().tiso_fit_varlen(_ext.F32, y.data_ptr(), None, out.data_ptr(), None,
                                    off.data_ptr(), 2, 16, flags, 0.0, 0.0, None,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    got = out.cpu()
    want0 = oracle.isotonic(y[:10].cpu())
    want1 = oracle.isotonic(y[10:26].cpu())
    assert_values(got[:10], want0, 3.0)
    assert_values(got[10:26], want1, 3.0)
    assert (got[26:] == 123.0).all()


def test_max_len_over_the_limit_is_refused() -> None:
    y = torch.zeros(600, device="cuda")
    off = torch.tensor([0, 600], dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="512"):
        torchisotonic_b200.isotonic_varlen(y, off)
    with pytest.raises(RuntimeError, match="512"):
        _ext.isotonic_tiles_varlen(y, None, off, 600, True)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_gradients_against_the_oracle(dtype) -> None:
    g = torch.Generator().manual_seed(21)
    lengths = torch.randint(0, 513, (120,), generator=g).tolist()
    y, off, w = _ragged(lengths, g, dtype, weighted=True)
    c = torch.randn(y.shape, generator=g, dtype=dtype)
    yc, wc = y.cuda().requires_grad_(), w.cuda().requires_grad_()
    out = torchisotonic_b200.isotonic_varlen(yc, off.cuda(), wc, y_min=0.3, y_max=2.0)
    gy, gw = torch.autograd.grad((out * c.cuda()).sum(), (yc, wc))
    fit, st = _oracle_rows(y, off, w)  # unclipped fit and blocks
    oy = np.zeros(y.shape, dtype=y.numpy().dtype)
    ow = np.zeros(y.shape, dtype=y.numpy().dtype)
    o = off.tolist()
    for r in range(len(o) - 1):
        a, b = o[r], o[r + 1]
        if b == a:
            continue
        gy_r, gw_r = oracle.grad(fit[a:b][None].numpy(), st[a:b][None].numpy(), c[a:b][None].numpy(),
                                 w[a:b][None].numpy(), y[a:b][None].numpy(), y_min=0.3, y_max=2.0)
        oy[a:b], ow[a:b] = gy_r[0], gw_r[0]
    tol = 1e-9 if dtype == torch.float64 else 2e-5
    torch.testing.assert_close(gy.cpu(), torch.from_numpy(oy), rtol=tol, atol=tol)
    torch.testing.assert_close(gw.cpu(), torch.from_numpy(ow), rtol=tol, atol=tol * 10)


@pytest.mark.parametrize("max_len", [8, 13, 16, 30, 64])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16])
def test_short_ragged_gradients(max_len: int, dtype) -> None:
    # rows of at most 64 elements take the register backward (8 elements a lane, 1 to 8 lanes a
    # row): every length up to max_len, empty rows, a packed base offset that leaves rows off any
    # 16-byte boundary, weighted or not, with and without clip, against the oracle row by row
    g = torch.Generator().manual_seed(max_len)
    lengths = torch.randint(0, max_len + 1, (300,), generator=g).tolist()
    y, off, w = _ragged(lengths, g, dtype, weighted=True, base=3)
    c = torch.randn(y.shape, generator=g).to(dtype)
    acc = torch.float64 if dtype == torch.float64 else torch.float32
    tol = {torch.float64: 1e-9, torch.float32: 2e-5}.get(dtype, 2.0**-7)
    o = off.tolist()
    for ww in (w, None):
        # each case's own fit and blocks (the backward recomputes the block means from y and the
        # weights it is given, for the clip's mask), in the accumulation dtype as the kernels
        fit, st = _oracle_rows(y.to(acc), off, ww)
        for kw in ({}, {"y_min": 0.3, "y_max": 1.5}):
            gy, gw = _ext.isotonic_grad_varlen(st.cuda(), c.cuda(), None if ww is None else ww.cuda(),
                                               y.cuda(), off.cuda(), max_len, True, ww is not None,
                                               **kw)
            for r in range(len(o) - 1):
                a, b = o[r], o[r + 1]
                if a == b:
                    continue
                oy, ow = oracle.grad(fit[a:b][None].numpy(), st[a:b][None].numpy(),
                                     c[a:b][None].to(acc).numpy(),
                                     None if ww is None else ww[a:b][None].numpy(),
                                     y[a:b][None].to(acc).numpy(), **kw)
                torch.testing.assert_close(gy[a:b].cpu().double(),
                                           torch.from_numpy(oy[0]).to(dtype).double(),
                                           rtol=tol, atol=tol)
                if ww is not None:
                    torch.testing.assert_close(gw[a:b].cpu().double(),
                                               torch.from_numpy(ow[0]).double(),
                                               rtol=max(tol, 1e-6), atol=max(tol, 1e-6) * 4)


def test_short_ragged_gradients_rows_longer_than_the_lanes_hold() -> None:
    # a row longer than its lanes' capacity (8 lanes of 8 for max_len 64): its first 64 elements
    # are a row, the rest of its gradient untouched
    g = torch.Generator().manual_seed(12)
    y = torch.randn(100, generator=g, dtype=torch.float64)
    off = torch.tensor([0, 20, 100], dtype=torch.int64)
    st = torch.zeros(100, dtype=torch.bool)
    st[[0, 5, 20, 50, 90]] = True
    c = torch.randn(100, generator=g, dtype=torch.float64)
    gy, _ = _ext.isotonic_grad_varlen(st.cuda(), c.cuda(), None, None, off.cuda(), 64, True, False)
    got = gy.cpu()
    for a, b in ((0, 20), (20, 84)):
        oy, _ = oracle.grad(y[a:b][None].numpy(), st[a:b][None].numpy(), c[a:b][None].numpy())
        torch.testing.assert_close(got[a:b], torch.from_numpy(oy[0]), rtol=1e-12, atol=1e-12)


def test_c5_ragged_recipe_packed_equals_padded() -> None:
    # The benchmark's quantile head with ragged rows (bf16 [4096, 64], 10% of rows of length
    # L ~ randint(16, 64) padded at the end with the row's max + 1): fitting the packed rows gives
    # exactly the padded batch's fit and gradients on the valid elements.
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    b = 4096
    base = (torch.cumsum(0.1 + torch.randn(b, 64, generator=gen, device=dev), 1)
            + 0.3 * torch.randn(b, 64, generator=gen, device=dev))
    ragged = torch.rand(b, generator=gen, device=dev) < 0.1
    lengths = torch.where(ragged, torch.randint(16, 64, (b,), generator=gen, device=dev),
                          torch.full((b,), 64, device=dev))
    pos = torch.arange(64, device=dev)[None]
    valid = pos < lengths[:, None]
    rowmax = torch.where(valid, base, torch.tensor(-math.inf, device=dev)).amax(1)
    padded = torch.where(valid, base, (rowmax + 1)[:, None].expand(-1, 64)).bfloat16()
    w = 0.1 + torch.rand(b, 64, generator=gen, device=dev)
    up = torch.randn(b, 64, generator=gen, device=dev).bfloat16()
    yp = padded.clone().requires_grad_()
    wp = w.clone().requires_grad_()
    fp = torchisotonic_b200.isotonic(yp, wp)
    gyp, gwp = torch.autograd.grad((fp * up).sum(), (yp, wp))
    packed = padded[valid]
    off = torch.zeros(b + 1, dtype=torch.int64, device=dev)
    off[1:] = torch.cumsum(lengths, 0)
    yv = packed.clone().requires_grad_()
    wv = w[valid].clone().requires_grad_()
    fv = torchisotonic_b200.isotonic_varlen(yv, off, wv, max_len=64)
    gyv, gwv = torch.autograd.grad((fv * up[valid]).sum(), (yv, wv))
    assert torch.equal(fv, fp[valid])
    torch.testing.assert_close(gyv.float(), gyp[valid].float(), rtol=0, atol=0)
    torch.testing.assert_close(gwv, gwp[valid], rtol=1e-6, atol=1e-6)


def test_the_c_abi_directly() -> None:
    g = torch.Generator().manual_seed(4)
    lengths = [5, 0, 100, 512, 1]
    y, off, w = _ragged(lengths, g, torch.float64, weighted=True)
    yc, wc, offc = y.cuda(), w.cuda(), off.cuda()
    out = torch.empty_like(yc)
    starts = torch.empty(yc.shape, dtype=torch.bool, device="cuda")
    bad = torch.empty(1, dtype=torch.int32, device="cuda")
    so = _ext.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rc = so.tiso_fit_varlen(_ext.F64, yc.data_ptr(), wc.data_ptr(), out.data_ptr(),
                            starts.data_ptr(), offc.data_ptr(), len(lengths), 512,
                            _ext.INCREASING | _ext.EXACT, 0.0, 0.0, bad.data_ptr(), stream)
    assert rc == 0, so.tiso_last_error()
    want, wst = _oracle_rows(y, off, w)
    assert_values(out.cpu(), want, scale_of(y))
    assert torch.equal(starts.cpu(), wst)
    assert int(bad.item()) == 0
    gup = torch.randn(y.shape, generator=g, dtype=torch.float64).cuda()
    gy = torch.empty_like(yc)
    gw = torch.empty_like(wc)
    rc = so.tiso_grad_varlen(_ext.F64, yc.data_ptr(), wc.data_ptr(), starts.data_ptr(),
                             gup.data_ptr(), gy.data_ptr(), gw.data_ptr(), offc.data_ptr(),
                             len(lengths), 512, _ext.WANT_GRAD_W, 0.0, 0.0, stream)
    assert rc == 0, so.tiso_last_error()
    o = off.tolist()
    for r in range(len(lengths)):
        a, b = o[r], o[r + 1]
        if a == b:
            continue
        oy, ow = oracle.grad(want[a:b][None].numpy(), wst[a:b][None].numpy(),
                             gup[a:b][None].cpu().numpy(), w[a:b][None].numpy(), y[a:b][None].numpy())
        np.testing.assert_allclose(gy[a:b].cpu().numpy(), oy[0], rtol=1e-9, atol=1e-9)
        np.testing.assert_allclose(gw[a:b].cpu().numpy(), ow[0], rtol=1e-9, atol=1e-9)
    # a non-positive weight is reported
    wc[3] = 0.0
    rc = so.tiso_fit_varlen(_ext.F64, yc.data_ptr(), wc.data_ptr(), out.data_ptr(), None,
                            offc.data_ptr(), len(lengths), 512, _ext.INCREASING | _ext.EXACT,
                            0.0, 0.0, bad.data_ptr(), stream)
    assert rc == 0 and int(bad.item()) == 1
