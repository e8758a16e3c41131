"""Backward parity on the GPU: gradients through the public API against the oracle's block
sums (the reference's CPU backward, src/torchisotonic/_api.py:86-115, restated in
oracle/pava.c), the reference's own gradient tests (tests/test_grad.py,
tests/test_cuda.py:137-221), the golden fixtures, and the fwd+bwd benchmark configs."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from conftest import golden_case, golden_names
from golden_util import DTYPES, tensor
from test_fit_gpu import PATTERNS, c3, c4, c5, pattern
from torch.autograd import gradcheck

import oracle
import torchisotonic_b200
from torchisotonic_b200 import _ext

pytestmark = pytest.mark.gpu


def grads_cuda(y, w, c, **kw):
    yy = y.cuda().requires_grad_()
    ins = [yy]
    ww = None
    if w is not None:
        ww = w.cuda().requires_grad_()
        ins.append(ww)
    loss = (torchisotonic_b200.isotonic(yy, ww, **kw) * c.cuda()).sum()
    gs = torch.autograd.grad(loss, ins)
    return gs[0].cpu(), (gs[1].cpu() if w is not None else None)


def grads_oracle(y, w, c, increasing=True, y_min=None, y_max=None):
    """The oracle's gradients of sum(isotonic(y, w) * c) for [batch, n] rows."""
    acc = torch.float64 if y.dtype == torch.float64 else torch.float32
    fy = y.to(acc).numpy()
    fw = None if w is None else w.to(acc).numpy()
    fit, starts = oracle.fit(fy, fw, increasing=increasing)
    gy, gw = oracle.grad(fit, starts, c.to(acc).numpy(), fw, fy if w is not None else None,
                         y_min=y_min, y_max=y_max)
    return torch.from_numpy(gy), None if gw is None else torch.from_numpy(gw)


def check_grads(y, w, c, tol=1e-9, **kw):
    gy, gw = grads_cuda(y, w, c, **kw)
    kw.pop("dim", None)
    oy, ow = grads_oracle(y, w, c, **kw)
    scale = 1 + float(y.double().nan_to_num(0.0).abs().max())
    torch.testing.assert_close(gy.double(), oy.double().to(gy.dtype).double(), rtol=tol,
                               atol=tol, equal_nan=True)
    if w is not None:
        torch.testing.assert_close(gw.double(), ow.double(), rtol=tol, atol=tol * scale,
                                   equal_nan=True)


@pytest.mark.parametrize("name", golden_names(lambda k, m: m["grad"]))
def test_golden_gradients(name: str) -> None:
    case = golden_case(name)
    y = tensor(case["y"], case["dtype"])
    w = None
    if "w" in case:
        w = torch.from_numpy(np.array(case["w"]))
        if case["dtype"] in ("float32", "float64"):
            w = w.to(DTYPES[case["dtype"]])
    c = tensor(case["c"], case["dtype"])
    gy, gw = grads_cuda(y, w, c, **case["kwargs"])
    tol = {"float64": 1e-9, "float32": 1e-4}.get(case["dtype"], 1e-2)
    want_gy = tensor(case["gy"], case["dtype"])
    torch.testing.assert_close(gy.double(), want_gy.double(), rtol=tol, atol=tol)
    if w is not None:
        want_gw = torch.from_numpy(np.array(case["gw"]))
        scale = 1 + float(y.double().nan_to_num(0.0).abs().max())
        torch.testing.assert_close(gw.double(), want_gw.double(), rtol=tol, atol=tol * scale,
                                   equal_nan=True)


@pytest.mark.parametrize(
    ("batch", "n"),
    [(70, 31), (70, 32), (9, 33), (9, 64), (9, 65), (7, 128), (5, 512), (5, 513), (5, 1000),
     (5, 1024), (3, 1025), (3, 2048), (3, 2049), (3, 5000), (2, 70_000)],
)  # fmt: skip
def test_gradients_match_oracle(batch: int, n: int) -> None:
    # tests/test_cuda.py:137-157, plus multi-tile rows of the backward (n > 1024)
    g = torch.Generator().manual_seed(n)
    y = torch.linspace(0, 3, n, dtype=torch.float64) + torch.randn(batch, n, generator=g,
                                                                   dtype=torch.float64)
    w = torch.rand(batch, n, generator=g, dtype=torch.float64) + 0.1
    c = torch.randn(batch, n, generator=g, dtype=torch.float64)
    check_grads(y, w, c, increasing=False)
    check_grads(y, None, c)
    check_grads(y, w, c, y_min=0.5, y_max=2.5)
    check_grads(y.float(), w.float(), c.float(), tol=2e-5)


@pytest.mark.parametrize("name", PATTERNS)
@pytest.mark.parametrize("n", [1024, 1025, 3000, 70_000])
def test_gradient_blocks_across_tiles(name: str, n: int) -> None:
    # tests/test_cuda.py:160-183: the gradient is the block average over the blocks the GPU's
    # own fit reports, whatever the data.
    g = torch.Generator().manual_seed(n)
    y = pattern(name, n, g).expand(3, n).contiguous()
    w = torch.rand(3, n, generator=g, dtype=torch.float64) + 0.1
    c = torch.randn(3, n, generator=g, dtype=torch.float64)
    for weights in (w, None):
        gy, gw = grads_cuda(y, weights, c)
        _, starts = _ext.isotonic_tiles(y.cuda(), None if weights is None else weights.cuda(),
                                        True, True, True)
        ones = torch.ones_like(y) if weights is None else weights
        fit = torchisotonic_b200.isotonic(y.cuda(), None if weights is None else weights.cuda())
        ogy, ogw = oracle.grad(fit.cpu().numpy(), starts.cpu().numpy(), c.numpy(),
                               ones.numpy(), y.numpy() if weights is not None else None)
        torch.testing.assert_close(gy, torch.from_numpy(ogy), rtol=1e-9, atol=1e-9)
        if weights is not None:
            scale = 1e-9 * (1 + float(y.abs().max()))
            torch.testing.assert_close(gw, torch.from_numpy(ogw), rtol=1e-9, atol=scale)


@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("kwargs", [{}, {"increasing": False}, {"y_min": -0.3, "y_max": 0.5},
                                    {"dim": 0}])
def test_matches_finite_differences(seed: int, kwargs: dict) -> None:
    # tests/test_grad.py:21-29
    g = torch.Generator().manual_seed(seed)
    y = torch.randn(4, 13, generator=g, dtype=torch.float64).cuda().requires_grad_()
    w = (torch.rand(4, 13, generator=g, dtype=torch.float64) + 0.1).cuda().requires_grad_()
    assert gradcheck(lambda y, w: torchisotonic_b200.isotonic(y, w, **kwargs), (y, w))
    assert gradcheck(lambda y: torchisotonic_b200.isotonic(y, **kwargs), (y,))


def test_block_average_and_close_values() -> None:
    # tests/test_grad.py:32-56
    y = torch.tensor([3.0, 1.0, 2.0], device="cuda", requires_grad=True)
    c = torch.tensor([1.0, 2.0, 6.0], device="cuda")
    (grad,) = torch.autograd.grad((torchisotonic_b200.isotonic(y) * c).sum(), (y,))
    torch.testing.assert_close(grad.cpu(), torch.full((3,), 3.0))
    one = torch.tensor(1.0).view(torch.int32)
    rows = [(one + torch.arange(1000, dtype=torch.int32)).view(torch.float32)[None],
            torch.linspace(0, 1, 10**6)[None]]
    for row in rows:
        for batch in (1, 3):
            yy = row.expand(batch, -1).contiguous().cuda().requires_grad_()
            cc = torch.randn(yy.shape, generator=torch.Generator().manual_seed(batch)).cuda()
            out = torchisotonic_b200.isotonic(yy)
            assert torch.equal(out, yy)
            (gr,) = torch.autograd.grad((out * cc).sum(), (yy,))
            assert torch.equal(gr, cc)


def test_weights_alone_broadcast_and_dtypes() -> None:
    y = torch.randn(3, 8, dtype=torch.float64, device="cuda")
    w = (torch.rand(8, dtype=torch.float64) + 0.1).cuda().requires_grad_()
    assert gradcheck(lambda w: torchisotonic_b200.isotonic(y, w), (w,))
    yy = torch.randn(2, 50, device="cuda", requires_grad=True)
    (grad,) = torch.autograd.grad(torchisotonic_b200.isotonic(yy).sum(), (yy,))
    assert grad.dtype == torch.float32
    assert not torchisotonic_b200.isotonic(torch.randn(2, 5, device="cuda")).requires_grad


def test_nan_row_gradients() -> None:
    # The CPU convention (src/torchisotonic/csrc/pava.h:30-37): a NaN row is one block, so
    # d/dy = w G / W is finite and d/dw is NaN.
    for n in (50, 5000):
        y = torch.randn(4, n, dtype=torch.float64, generator=torch.Generator().manual_seed(n))
        y[1, 7] = math.nan
        w = torch.rand(4, n, dtype=torch.float64) + 0.1
        c = torch.randn(4, n, dtype=torch.float64)
        check_grads(y, w, c)


def test_config_c3_fwd_bwd_slice() -> None:
    y, w = c3(16, seed=1)
    c = torch.randn(y.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(2))
    check_grads(y, w, c, y_min=0.0, y_max=1.0)


def test_config_c5_fwd_bwd() -> None:
    # the differentiable quantile head: bf16 y, float32 w, upstream N(0, 1), ragged rows
    y, w = c5(65536)
    c = torch.randn(y.shape, generator=torch.Generator().manual_seed(3)).bfloat16()
    gy, gw = grads_cuda(y, w, c)
    oy, ow = grads_oracle(y, w, c)
    torch.testing.assert_close(gy.double(), oy.bfloat16().double(), rtol=2**-8, atol=1e-3)
    scale = 1 + float(y.double().abs().max())
    torch.testing.assert_close(gw.double(), ow.double(), rtol=1e-4, atol=1e-5 * scale)


@pytest.mark.parametrize("n", [1_100_000, 3_000_000])
def test_long_rows_scanned_in_chunks(n: int) -> None:
    # rows of more than 1024 tiles of 1024 elements: the scan of tile sums runs in chunks of
    # 256 tiles on many CTAs; blocks span many tiles and chunks
    g = torch.Generator().manual_seed(n)
    i = torch.arange(n, dtype=torch.float64)
    y = torch.stack([torch.sin(i / 50_000) + 0.3 * torch.randn(n, generator=g, dtype=torch.float64),
                     (i % 300_000) * 1e-6 + 0.01 * torch.randn(n, generator=g, dtype=torch.float64)])
    w = torch.rand(2, n, generator=g, dtype=torch.float64) + 0.1
    c = torch.randn(2, n, generator=g, dtype=torch.float64)
    check_grads(y, w, c)
    check_grads(y, None, c, y_min=-0.5, y_max=0.5)


def test_config_c4_fwd_bwd() -> None:
    # one row of 1e8 (97,657 tiles, 382 chunks: the scan over chunks takes two pieces)
    y, w = c4(100_000_000)
    c = torch.randn(y.shape, generator=torch.Generator().manual_seed(4))
    check_grads(y.cpu(), w.cpu(), c, tol=2e-5)
