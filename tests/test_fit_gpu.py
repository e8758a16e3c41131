"""Forward parity on the GPU: the public API (torchisotonic_b200.isotonic, which calls the C ABI
of include/tiso.h) against the oracle, over the reference's own test cases
(tests/test_cuda.py, tests/test_isotonic.py), the golden fixtures, and the benchmark configs."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from conftest import golden_case, golden_names
from golden_util import DTYPES, out_tensor, tensor
from parity import assert_values, check_fit, check_starts, kkt_check, scale_of

import oracle
import torchisotonic_b200
from torchisotonic_b200 import _ext

pytestmark = pytest.mark.gpu


def _golden_inputs(case: dict):
    y = tensor(case["y"], case["dtype"])
    w = None
    if "w" in case:
        w = torch.from_numpy(np.array(case["w"]))
        if case["dtype"] in ("float32", "float64"):
            w = w.to(DTYPES[case["dtype"]])
    return y, w, dict(case["kwargs"])


@pytest.mark.parametrize("name", golden_names())
def test_golden_fixtures(name: str) -> None:
    # Against the reference's own CPU outputs, at the reference's GPU-vs-CPU tolerances
    # (tests/test_cuda.py:27); and against the extended-precision oracle at the tight ones.
    case = golden_case(name)
    y, w, kw = _golden_inputs(case)
    got = torchisotonic_b200.isotonic(y.cuda(), None if w is None else w.cuda(), **kw).cpu()
    want = out_tensor(case)
    assert got.dtype == want.dtype and got.shape == want.shape
    tol = {"float64": 1e-12, "float32": 1e-4}.get(case["dtype"], 1e-2)
    sc = scale_of(y) if case["dtype"] == "float64" else 1.0
    torch.testing.assert_close(got.double(), want.double(), rtol=tol, atol=tol * sc,
                               equal_nan=True)
    if y.numel():
        assert_values(got, oracle.isotonic(y, w, **kw), scale_of(y))


@pytest.mark.parametrize("batch", [1, 3, 127, 128, 129, 5000])
@pytest.mark.parametrize("n", [1, 2, 7, 100, 1000])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_matches_oracle_grid(batch: int, n: int, dtype: torch.dtype) -> None:
    # tests/test_cuda.py:31-40
    g = torch.Generator().manual_seed(batch * 1000 + n)
    y = torch.linspace(0, 3, n, dtype=dtype) + torch.randn(batch, n, generator=g, dtype=dtype)
    w = (torch.rand(batch, n, generator=g) + 0.1).to(dtype)
    check_fit(y)
    check_fit(y, w)
    check_fit(y, w, increasing=False, y_min=-0.5, y_max=2.0)


TILE_SHAPES = [1, 2, 15, 16, 17, 31, 32, 33, 64, 100, 128, 255, 256, 257, 511, 512, 513, 1000,
               1023, 1024, 1025, 2047, 2048, 2049, 4095, 4096, 4097, 6143, 6145, 8192, 8193,
               12289, 65537, 100_000]


@pytest.mark.parametrize("n", TILE_SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 70])
def test_tile_shapes(n: int, batch: int) -> None:
    # tests/test_cuda.py:65-81: every thread, segment and tile edge; one and many tiles.
    if batch * n > 2_000_000:
        batch = max(1, 2_000_000 // n)
    g = torch.Generator().manual_seed(n + batch)
    y = torch.linspace(0, 3, n, dtype=torch.float64) + torch.randn(batch, n, generator=g,
                                                                   dtype=torch.float64)
    w = (torch.rand(batch, n, generator=g) + 0.1).double()
    check_fit(y)
    check_fit(y, w, increasing=False)
    check_fit(y.float())
    check_fit(y.float(), w.float())


PATTERNS = ["increasing", "decreasing", "saw", "cliff", "walk", "constant", "valley"]


def pattern(name: str, n: int, g: torch.Generator) -> torch.Tensor:
    # tests/test_cuda.py:108-122
    i = torch.arange(n, dtype=torch.float64)
    if name == "increasing":
        return i
    if name == "decreasing":
        return -i
    if name == "saw":
        return i % 7 + (i % 1500) * 0.1
    if name == "cliff":
        return torch.where(i == n - 1, torch.tensor(-1e9, dtype=torch.float64), i)
    if name == "walk":
        return torch.randn(n, generator=g, dtype=torch.float64).cumsum(0)
    if name == "constant":
        return torch.ones(n, dtype=torch.float64)
    return (i - n / 3) ** 2


@pytest.mark.parametrize("name", PATTERNS)
@pytest.mark.parametrize("n", [700, 1025, 3000, 5000, 9000, 70_000])
def test_patterns(name: str, n: int) -> None:
    # tests/test_cuda.py:125-134. float32-representable weights keep w y exact, so that the
    # exact ties of the constant pattern are ties in the kernels' arithmetic too.
    g = torch.Generator().manual_seed(n)
    y = pattern(name, n, g)[None]
    w = (torch.rand(1, n, generator=g) + 0.1).double()
    check_fit(y)
    check_fit(y, w)
    check_fit(y, w, increasing=False)
    check_fit(y.float())


def test_nan_rows() -> None:
    # tests/test_cuda.py:51-55, whole rows and tiled rows
    for n in (50, 9000):
        y = torch.randn(30, n, dtype=torch.float64, generator=torch.Generator().manual_seed(n))
        y[7, 3] = math.nan
        y[29, n - 1] = math.nan
        y[11, n // 2] = math.nan
        check_fit(y)
        check_fit(y.float())


def test_other_dims_and_low_precision() -> None:
    # tests/test_cuda.py:58-62
    y = torch.randn(4, 60, 5, generator=torch.Generator().manual_seed(1))
    for t in (y, y.half(), y.bfloat16()):
        check_fit(t, dim=1)
        check_fit(t, dim=0, increasing=False)


@pytest.mark.parametrize("n", [100, 1000, 5000, 100_000])
@pytest.mark.parametrize("weighted", [False, True])
def test_exact_flag(n: int, weighted: bool) -> None:
    # tests/test_cuda.py:84-102: exact=True is the default; exact=False changes float32 only.
    g = torch.Generator().manual_seed(n)
    y = torch.linspace(0, 3, n, dtype=torch.float64) + torch.randn(8, n, generator=g,
                                                                   dtype=torch.float64)
    w = torch.rand(8, n, generator=g, dtype=torch.float64) + 0.1 if weighted else None
    yc, wc = y.cuda(), None if w is None else w.cuda()
    for dtype in (torch.float32, torch.float64):
        wd = None if wc is None else wc.to(dtype)
        default = torchisotonic_b200.isotonic(yc.to(dtype), wd)
        assert torch.equal(default, torchisotonic_b200.isotonic(yc.to(dtype), wd, exact=True))
        fast = torchisotonic_b200.isotonic(yc.to(dtype), wd, exact=False)
        if dtype == torch.float64:
            assert torch.equal(fast, default)
    check_fit(y.float(), None if w is None else w.float(), exact=False)


@pytest.mark.parametrize("name", ["collinear", "offset", "consecutive"])
@pytest.mark.parametrize("n", [1000, 100_000])
def test_float32_fit_is_monotone(name: str, n: int) -> None:
    # tests/test_cuda.py:224-240
    g = torch.Generator().manual_seed(n)
    i = torch.arange(n, dtype=torch.float64)
    one = torch.tensor(1.0).view(torch.int32)
    y = {
        "collinear": 1e6 + 1e-3 * i + 1e-9 * torch.randn(n, generator=g, dtype=torch.float64),
        "offset": 1e6 + torch.randn(n, generator=g, dtype=torch.float64),
        "consecutive": (one + torch.arange(n, dtype=torch.int32)).view(torch.float32).double(),
    }[name].float()
    u = torch.rand(n, generator=g)
    for w in (None, u + 0.1, torch.exp(8 * u)):
        fit = torchisotonic_b200.isotonic(y.cuda(), None if w is None else w.cuda())
        assert bool((fit[1:] >= fit[:-1]).all())
        check_fit(y[None], None if w is None else w[None])


@pytest.mark.parametrize("big", [1e3, 1e6, 1e12])
@pytest.mark.parametrize("n", [500, 3000, 100_000])
def test_cancelling_sums(n: int, big: float) -> None:
    # tests/test_cuda.py:243-265, at the reference's tolerances
    g = torch.Generator().manual_seed(n)
    k = torch.arange(n) % 64
    y = torch.where(k < 32, big, 1.0).double()
    y[k == 32] = -32 * big
    y += 1e-3 * (-1.0) ** k * (k > 32) + 1e-6 * torch.randn(n, generator=g, dtype=torch.float64)
    for w in (None, torch.rand(n, generator=g, dtype=torch.float64) + 0.1):
        for dtype, step, dev in ((torch.float64, 8 * 2.0**-52, 1e-14), (torch.float32, 0, 1e-7)):
            yy = y.to(dtype)[None]
            ww = None if w is None else w.to(dtype)[None]
            want = oracle.isotonic(yy.double(), None if ww is None else ww.double())
            got = torchisotonic_b200.isotonic(yy.cuda(), None if ww is None else ww.cuda())
            got = got.double().cpu()
            scale = float(yy.double().abs().max())
            assert float((got[:, :-1] - got[:, 1:]).max()) <= step * scale
            torch.testing.assert_close(got, want, rtol=0, atol=dev * scale)


def test_known_answers_and_errors() -> None:
    for dt in (torch.float16, torch.bfloat16, torch.float32, torch.float64):
        got = torchisotonic_b200.isotonic(torch.tensor([3.0, 1.0, 2.0, 5.0], dtype=dt).cuda())
        assert got.dtype == dt
        assert got.double().cpu().tolist() == [2.0, 2.0, 2.0, 5.0]
    got = torchisotonic_b200.isotonic(torch.tensor([3, 1, 2]).cuda())
    assert got.dtype == torch.get_default_dtype() and got.cpu().tolist() == [2.0, 2.0, 2.0]
    _, st = _ext.isotonic_tiles(torch.tensor([[1.0, 2.0, 2.0, 3.0]]).cuda(), None, True, True,
                                True)
    assert st.cpu().tolist() == [[True, True, False, True]]
    with pytest.raises(ValueError, match="strictly positive"):
        torchisotonic_b200.isotonic(torch.zeros(3).cuda(), torch.tensor([1.0, 0.0, 1.0]).cuda())
    with pytest.raises(ValueError, match="strictly positive"):
        torchisotonic_b200.isotonic(torch.zeros(2, 9000).cuda(), torch.full((9000,), -1.0).cuda())
    with pytest.raises(ValueError, match="does not fit y"):
        torchisotonic_b200.isotonic(torch.zeros(3).cuda(), torch.ones(4).cuda())


# ---- the benchmark configs: the oracle on a slice, size-independent checks on all of it ----


def c1(batch: int = 1000) -> torch.Tensor:
    g = torch.Generator().manual_seed(0)
    return 0.001 * torch.arange(5000) + torch.randn(batch, 5000, generator=g)


def test_config_c1() -> None:
    y = c1()
    check_fit(y)
    out, st = _ext.isotonic_tiles(y.cuda(), None, True, True, True)
    kkt_check(y.cuda(), None, out, st)


@pytest.mark.parametrize("exact", [True, False])
def test_config_c2(exact: bool) -> None:
    g = torch.Generator().manual_seed(0)
    y = -0.1 * torch.arange(16) + 0.5 * torch.randn(1_000_000, 16, generator=g)
    check_fit(y, increasing=False, exact=exact)
    out, st = _ext.isotonic_tiles(y.cuda(), None, False, exact, True)
    if exact:
        kkt_check(y.cuda(), None, out, st, increasing=False)


def c3(batch: int, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    n = 65536
    y = torch.sigmoid(torch.linspace(-4, 4, n, dtype=torch.float64)
                      + torch.randn(batch, n, generator=g, dtype=torch.float64))
    w = torch.empty(batch, n, dtype=torch.float64).exponential_(1.0, generator=g) + 0.1
    rows = (torch.rand(batch, generator=g) < 0.01).nonzero().squeeze(1)
    y[rows, torch.randint(n, (len(rows),), generator=g)] = math.nan
    y[0, 12345] = math.nan  # at least one NaN row in any slice
    return y, w


def test_config_c3_slice() -> None:
    y, w = c3(48)
    check_fit(y, w, y_min=0.0, y_max=1.0)
    check_fit(y, w)


def test_config_c3_full() -> None:
    y, w = c3(4096)
    yc, wc = y.cuda(), w.cuda()
    del y, w
    out, st = _ext.isotonic_tiles(yc, wc, True, True, True)
    kkt_check(yc, wc, out, st)
    clipped = torchisotonic_b200.isotonic(yc, wc, y_min=0.0, y_max=1.0)
    assert torch.equal(clipped.nan_to_num(-7.0), out.clamp(0.0, 1.0).nan_to_num(-7.0))


def c4(n: int, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    z = torch.randn(n, generator=g, device="cuda").sort().values
    w = (1 + torch.poisson(torch.full((n,), 0.5, device="cuda"), generator=g)).float()
    y = (torch.binomial(w, torch.sigmoid(3 * z), generator=g) / w).float()
    return y[None], w[None]


def test_config_c4_slice() -> None:
    y, w = c4(3_000_000)
    check_fit(y.cpu(), w.cpu())


def test_config_c4_full() -> None:
    y, w = c4(100_000_000)
    out, st = _ext.isotonic_tiles(y, w, True, True, True)
    kkt_check(y, w, out, st, rel=1e-9)
    assert bool((out[0, 1:] >= out[0, :-1]).all())


def c5(batch: int, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    base = torch.cumsum(0.1 + torch.randn(batch, 64, generator=g), 1) + 0.3 * torch.randn(
        batch, 64, generator=g)
    ragged = torch.rand(batch, generator=g) < 0.1
    lengths = torch.randint(16, 64, (batch,), generator=g)
    pos = torch.arange(64)[None]
    pad = ragged[:, None] & (pos >= lengths[:, None])
    rowmax = torch.where(pos < lengths[:, None], base, torch.tensor(-math.inf)).amax(1)
    base = torch.where(pad, (rowmax + 1)[:, None].expand(-1, 64), base)
    w = 0.1 + torch.rand(batch, 64, generator=g)
    return base.bfloat16(), w


def test_config_c5_forward() -> None:
    y, w = c5(65536)
    check_fit(y, w)
