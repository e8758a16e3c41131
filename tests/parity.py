"""Parity helpers: the CUDA path against the oracle, and size-independent checks of a fit.

Tolerances (the bar of the reference's own tests, src tests/test_cuda.py:18-28, tightened
where the kernels' arithmetic allows):
  float64            rtol = 1e-12, atol = 1e-12 x data scale;
  float32 exact=True within 2 units in the last place (the oracle and the kernels round
                     the same quotient; double rounding may cost one);
  float32 exact=False within 1e-3 x data scale (the reference's stated band);
  float16/bfloat16   one unit in the last place of the output dtype.
Block starts: identical to the extended-precision oracle's.
"""

from __future__ import annotations

import numpy as np
import torch

import oracle
import torchisotonic_b200
from torchisotonic_b200 import _ext

TOL = {torch.float64: 1e-12}


def scale_of(y: torch.Tensor) -> float:
    if y.numel() == 0:
        return 1.0
    return max(1.0, float(y.double().nan_to_num(0.0, 0.0, 0.0).abs().max()))


def assert_values(got: torch.Tensor, want: torch.Tensor, scale: float, exact: bool = True) -> None:
    got = got.cpu()
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert torch.equal(got.isnan(), want.isnan())
    g, w = got.double().nan_to_num(0.0), want.double().nan_to_num(0.0)
    if got.dtype == torch.float64:
        torch.testing.assert_close(g, w, rtol=1e-12, atol=1e-12 * scale)
    elif got.dtype == torch.float32:
        if exact:
            torch.testing.assert_close(g, w, rtol=2.4e-7, atol=4 * 2.0**-24 * scale)
        else:
            torch.testing.assert_close(g, w, rtol=1e-3, atol=1e-3 * scale)
    else:
        eps = 2.0**-8 if got.dtype == torch.bfloat16 else 2.0**-11
        torch.testing.assert_close(g, w, rtol=eps, atol=eps * 1e-3)


def fit_both(y: torch.Tensor, w: torch.Tensor | None = None, **kw):
    """(CUDA result, oracle result) of torchisotonic.isotonic(y, w, **kw); y, w on the CPU."""
    got = torchisotonic_b200.isotonic(y.cuda(), None if w is None else w.cuda(), **kw)
    kw.pop("exact", None)  # the oracle is exact
    want = oracle.isotonic(y, w, **kw)
    return got, want


def check_fit(y: torch.Tensor, w: torch.Tensor | None = None, starts: bool = True,
              exact: bool = True, **kw) -> None:
    """The public API on CUDA against the oracle: values, and the block starts."""
    got, want = fit_both(y, w, exact=exact, **kw)
    assert got.is_cuda and got.shape == want.shape
    assert_values(got, want, scale_of(y), exact)
    if starts and exact and y.numel():
        check_starts(y, w, increasing=kw.get("increasing", True), dim=kw.get("dim", -1))


def check_starts(y: torch.Tensor, w: torch.Tensor | None, increasing: bool = True,
                 dim: int = -1) -> None:
    out_dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
    acc = _ext.acc_dtype(out_dtype)
    rows = y.movedim(dim, -1)
    flat = rows.reshape(-1, rows.shape[-1]).to(out_dtype).contiguous()
    fw = None
    if w is not None:
        fw = w.to(acc).broadcast_to(y.shape).movedim(dim, -1).reshape(flat.shape).contiguous()
    _, st = _ext.isotonic_tiles(flat.cuda(), None if fw is None else fw.cuda(), increasing,
                                True, True)
    yo = flat.to(acc).numpy()
    _, want = oracle.fit(yo, None if fw is None else fw.numpy(), increasing=increasing)
    got = st.cpu().numpy()
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        raise AssertionError(f"block starts differ at {len(bad)} places, first {bad[:5].tolist()}")


def kkt_check(y: torch.Tensor, w: torch.Tensor | None, out: torch.Tensor, starts: torch.Tensor,
              increasing: bool = True, rel: float = 1e-9) -> None:
    """Size-independent check of an unclipped fit of [batch, n] rows, on the GPU in float64.

    The isotonic regression is the unique x with: x monotone; x constant on its blocks, each
    the weighted mean of y over the block; and every prefix of a block with a weighted mean not
    below the block's (no block could be split). NaN rows: all NaN, one block at 0.
    """
    y = y.double()
    s = 1.0 if increasing else -1.0
    yy = s * y
    ww = torch.ones_like(y) if w is None else w.double()
    o = s * out.double()
    batch, n = y.shape
    nan_row = y.isnan().any(1)
    st = starts.clone()
    assert bool(st[:, 0].all()), "a block starts at every row's first element"
    assert bool(o[nan_row].isnan().all()), "NaN rows are NaN"
    assert bool((st[nan_row, 1:] == 0).all()), "NaN rows are one block"
    ok = ~nan_row
    yy, ww, o, st = yy[ok], ww[ok], o[ok], st[ok]
    if yy.numel() == 0:
        return
    scale = max(1.0, float(yy.abs().max()))
    # block ids over the flattened rows
    ids = st.reshape(-1).long().cumsum(0) - 1
    nblk = int(ids[-1]) + 1
    wsum = torch.zeros(nblk, dtype=torch.float64, device=y.device).index_add_(0, ids, ww.reshape(-1))
    tsum = torch.zeros(nblk, dtype=torch.float64, device=y.device).index_add_(
        0, ids, (ww * yy).reshape(-1))
    mean = tsum / wsum
    # values are the block means
    err = (o.reshape(-1) - mean[ids]).abs().max()
    assert float(err) <= rel * scale + 1e-6 * scale * (out.dtype != torch.float64), float(err)
    # consecutive blocks within a row strictly increase (in float64 of the sums)
    first = st.reshape(-1).nonzero().squeeze(1)
    row_of_block = first // n
    same_row = row_of_block[1:] == row_of_block[:-1]
    step = mean[1:] - mean[:-1]
    assert bool((step[same_row] > -rel * scale).all()), "block means must increase"
    # no block can be split: prefix sums of w (y - mean) within each block are >= 0
    dev = ww.reshape(-1) * (yy.reshape(-1) - mean[ids])
    c = dev.cumsum(0)
    start_c = (c - dev)[first]  # cumulative sum before each block's first element
    within = c - start_c[ids]
    wf = ww.reshape(-1)
    wc = wf.cumsum(0)
    wprefix = wc - (wc - wf)[first][ids]  # weight of the block's prefix up to each element
    tol = rel * scale * (1 + wprefix)
    assert bool((within >= -tol).all()), "a prefix of a block has a lower mean than the block"
