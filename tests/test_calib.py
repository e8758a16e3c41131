"""Calibration around the fit: fit_calibration (sort, pool equal scores, fit) and calibrate
(searchsorted + lerp), the reference's recipe of README.md:43-56.

CPU: the numpy oracle against the fixtures that the reference's own recipe produced
(tests/golden/make_calib_golden.py), the argument checks. GPU: the kernels against those
fixtures and the oracle. Bars: xs and the counts bit-exact; means and fit within float64's
1e-12 (labels summed in another order); calibrated values bit-exact on a given curve (the
kernel rounds every step as torch does); at sizes beyond the oracle, properties that hold
whatever the size: xs strictly increasing, counts summing to n, label sums kept by the fit.
"""

from __future__ import annotations

import json
import math
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import torchisotonic_b200
from torchisotonic_b200 import _ext

CALIB = Path(__file__).resolve().parent / "golden" / "calib.npz"


@lru_cache(maxsize=1)
def fixtures() -> dict[str, dict[str, np.ndarray]]:
    z = np.load(CALIB)
    meta = json.loads(bytes(z["__meta__"]).decode())
    return {name: {k: z[f"{name}/{k}"] for k in ("scores", "labels", "xs", "fit", "x", "read")}
            for name in meta}


NAMES = sorted(fixtures())


# ---------------------------------------------------------------------------------------------
# CPU: the oracle pinned to the reference, argument checks


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_recipe(name: str) -> None:
    c = fixtures()[name]
    xs, fit = oracle.fit_calibration(c["scores"], c["labels"])
    assert np.array_equal(xs, c["xs"])
    np.testing.assert_allclose(fit, c["fit"], rtol=1e-12, atol=1e-12)
    read = oracle.calibrate(c["x"], c["xs"], c["fit"])
    assert np.array_equal(read, c["read"], equal_nan=True)


def test_calibration_argument_checks() -> None:
    with pytest.raises(ValueError, match="one length"):
        torchisotonic_b200.fit_calibration(torch.zeros(3), torch.zeros(4))
    with pytest.raises(ValueError, match="1-D"):
        torchisotonic_b200.fit_calibration(torch.zeros(2, 3), torch.zeros(2, 3))
    with pytest.raises(TypeError):
        torchisotonic_b200.fit_calibration([1.0], torch.zeros(1))  # type: ignore[arg-type]
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torchisotonic_b200.fit_calibration(torch.zeros(3), torch.zeros(3))
    xs, fit = torchisotonic_b200.fit_calibration(torch.zeros(0), torch.zeros(0))
    assert xs.numel() == 0 and fit.numel() == 0 and fit.dtype == torch.float64
    with pytest.raises(ValueError, match="one length"):
        torchisotonic_b200.calibrate(torch.zeros(3), torch.zeros(2), torch.zeros(3))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torchisotonic_b200.calibrate(torch.zeros(3), torch.zeros(2), torch.zeros(2))


def test_calib_abi_checks() -> None:
    import ctypes

    so = _ext.lib()
    size = ctypes.c_size_t()
    assert so.tiso_calib_groups_workspace_size(_ext.F16, _ext.F32, 10, 0, ctypes.byref(size)) == 1
    assert b"key_dtype" in so.tiso_last_error()
    assert so.tiso_calib_groups_workspace_size(_ext.F32, _ext.F32, 0, 0, ctypes.byref(size)) == 1
    assert so.tiso_calib_interp(_ext.F32, None, 5, None, None, 0, None, None) == 1
    assert so.tiso_calib_interp(_ext.F32, None, 0, None, None, 3, None, None) == 0


# ---------------------------------------------------------------------------------------------
# GPU


def _cuda(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_fit_calibration_matches_reference(name: str) -> None:
    c = fixtures()[name]
    xs, fit = torchisotonic_b200.fit_calibration(_cuda(c["scores"]), _cuda(c["labels"]))
    assert xs.dtype == torch.from_numpy(c["scores"]).dtype and fit.dtype == torch.float64
    assert np.array_equal(xs.cpu().numpy(), c["xs"])
    np.testing.assert_allclose(fit.cpu().numpy(), c["fit"], rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_calibrate_matches_reference(name: str) -> None:
    c = fixtures()[name]
    got = torchisotonic_b200.calibrate(_cuda(c["x"]), _cuda(c["xs"]), _cuda(c["fit"]))
    assert got.dtype == torch.float64
    assert np.array_equal(got.cpu().numpy(), c["read"], equal_nan=True)


def _groups_oracle(s: np.ndarray, lab: np.ndarray):
    order = np.argsort(s, kind="stable")
    ss = s[order]
    head = np.ones(ss.size, dtype=bool)
    head[1:] = ss[1:] != ss[:-1]
    first = np.flatnonzero(head)
    counts = np.diff(np.append(first, ss.size))
    sums = np.add.reduceat(lab[order].astype(np.float64), first)
    return ss[first], sums / counts, counts.astype(np.float64)


def _scores(kind: str, n: int, gen: torch.Generator) -> torch.Tensor:
    if kind == "unique":
        return torch.sigmoid(torch.randn(n, generator=gen))
    if kind == "ties_many":
        return (torch.randint(0, 1000, (n,), generator=gen) / 1000).float()
    if kind == "ties_few":  # groups far longer than a tile
        return torch.randint(0, 3, (n,), generator=gen).float()
    if kind == "one":
        return torch.full((n,), 0.25)
    if kind == "sorted":
        return torch.arange(n, dtype=torch.float32)
    return -torch.arange(n, dtype=torch.float32)  # reversed


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["unique", "ties_many", "ties_few", "one", "sorted", "reversed"])
@pytest.mark.parametrize("n", [1, 15, 16, 17, 4095, 4096, 4097, 12289, 300_001])
def test_groups_against_oracle(kind: str, n: int) -> None:
    gen = torch.Generator().manual_seed(n + len(kind))
    s = _scores(kind, n, gen)
    lab = torch.bernoulli(torch.full((n,), 0.3), generator=gen)
    xs, y, w, groups = _ext.calib_groups(s.cuda(), lab.cuda())
    g, nan = groups.tolist()
    wx, wy, ww = _groups_oracle(s.numpy(), lab.numpy())
    assert nan == 0 and g == wx.size
    assert np.array_equal(xs[:g].cpu().numpy(), wx)
    assert np.array_equal(y[:g].cpu().numpy(), wy)  # 0/1 labels: sums exact, one rounding
    assert np.array_equal(w[:g].cpu().numpy(), ww)
    got_xs, got_fit = torchisotonic_b200.fit_calibration(s.cuda(), lab.cuda())
    want_xs, want_fit = oracle.fit_calibration(s.numpy(), lab.numpy())
    assert np.array_equal(got_xs.cpu().numpy(), want_xs)
    np.testing.assert_allclose(got_fit.cpu().numpy(), want_fit, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("key", [torch.float32, torch.float64, torch.float16, torch.int64])
@pytest.mark.parametrize("lab", [torch.bool, torch.int32, torch.float32, torch.float64])
def test_dtypes(key: torch.dtype, lab: torch.dtype) -> None:
    gen = torch.Generator().manual_seed(3)
    n = 20_000
    s = (torch.randn(n, generator=gen, dtype=torch.float64) * 100).round().to(key)
    raw = torch.bernoulli(torch.full((n,), 0.5, dtype=torch.float64), generator=gen)
    if lab == torch.float64:
        raw = torch.rand(n, generator=gen, dtype=torch.float64)
    labels = raw.to(lab)
    xs, fit = torchisotonic_b200.fit_calibration(s.cuda(), labels.cuda())
    assert xs.dtype == key
    key_np = s.double().numpy() if key in (torch.float16, torch.int64) else s.numpy()
    want_xs, want_fit = oracle.fit_calibration(key_np, labels.double().numpy())
    np.testing.assert_array_equal(xs.cpu().double().numpy(), want_xs.astype(np.float64))
    np.testing.assert_allclose(fit.cpu().numpy(), want_fit, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
def test_nan_scores_and_labels() -> None:
    s = torch.tensor([0.1, math.nan, 0.3], device="cuda")
    with pytest.raises(ValueError, match="NaN"):
        torchisotonic_b200.fit_calibration(s, torch.ones(3, device="cuda"))
    s = torch.tensor([0.1, 0.2, 0.3], device="cuda")
    lab = torch.tensor([1.0, math.nan, 0.0], device="cuda")
    xs, fit = torchisotonic_b200.fit_calibration(s, lab)
    assert xs.tolist() == pytest.approx([0.1, 0.2, 0.3]) and bool(fit.isnan().all())


@pytest.mark.gpu
def test_signed_zero_keeps_one_group() -> None:
    s = torch.tensor([0.0, -0.0, 1.0, -0.0], device="cuda")
    xs, fit = torchisotonic_b200.fit_calibration(s, torch.tensor([1.0, 0.0, 1.0, 0.0],
                                                                 device="cuda"))
    assert xs.tolist() == [0.0, 1.0] and fit.tolist() == pytest.approx([1 / 3, 1.0])


@pytest.mark.gpu
def test_calibrate_shapes_and_dtypes() -> None:
    gen = torch.Generator().manual_seed(4)
    s = torch.sigmoid(torch.randn(5000, generator=gen))
    lab = torch.bernoulli(s, generator=gen)
    xs, fit = torchisotonic_b200.fit_calibration(s.cuda(), lab.cuda())
    x = torch.rand(7, 9, generator=gen).cuda()
    got = torchisotonic_b200.calibrate(x, xs, fit)
    assert got.shape == (7, 9) and got.dtype == torch.float64
    want = oracle.calibrate(x.cpu().numpy().ravel(), xs.cpu().numpy(), fit.cpu().numpy())
    assert np.array_equal(got.cpu().numpy().ravel(), want)
    got32 = torchisotonic_b200.calibrate(x, xs, fit.float())
    assert got32.dtype == torch.float32
    # a curve of one point: constant, NaN where the interpolation divides 0 by 0
    one = torchisotonic_b200.calibrate(torch.tensor([0.0, 0.5, 1.0], device="cuda"),
                                       torch.tensor([0.5], device="cuda"),
                                       torch.tensor([0.7], dtype=torch.float64, device="cuda"))
    ref = oracle.calibrate(np.array([0.0, 0.5, 1.0], dtype=np.float32),
                           np.array([0.5], dtype=np.float32), np.array([0.7]))
    assert np.array_equal(one.cpu().numpy(), ref, equal_nan=True)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [20_000_000])
def test_large_properties(n: int) -> None:
    gen = torch.Generator(device="cuda").manual_seed(9)
    s = torch.sigmoid(torch.randn(n, generator=gen, device="cuda"))
    lab = torch.bernoulli(s, generator=gen)
    xs, y, w, groups = _ext.calib_groups(s, lab)
    g = int(groups[0])
    xs, y, w = xs[:g], y[:g], w[:g]
    assert bool((xs[1:] > xs[:-1]).all())
    assert int(w.sum()) == n
    assert float((y * w).sum()) == pytest.approx(float(lab.double().sum()), rel=1e-12)
    assert torch.equal(torch.unique(s), xs)
    got_xs, fit = torchisotonic_b200.fit_calibration(s, lab)
    assert torch.equal(got_xs, xs)
    assert bool((fit[1:] >= fit[:-1]).all())
    # the fit keeps every pooled block's label sum: so the total is kept
    assert float((fit * w).sum()) == pytest.approx(float(lab.double().sum()), rel=1e-10)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 4097, 100_003])
def test_presorted_pairs_are_read_in_place(n: int) -> None:
    gen = torch.Generator().manual_seed(n)
    s, _ = torch.sort((torch.randint(0, 50, (n,), generator=gen) / 7).float())
    lab = torch.rand(n, generator=gen, dtype=torch.float64)
    a = _ext.calib_groups(s.cuda(), lab.cuda())
    b = _ext.calib_groups(s.cuda(), lab.cuda(), presorted=True)
    g = int(a[3][0])
    assert int(b[3][0]) == g
    for x, y in zip(a[:3], b[:3]):
        assert torch.equal(x[:g], y[:g])


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["ties_few", "ties_many", "unique"])
def test_groups_across_scan_chunks(kind: str) -> None:
    # more than 4096 tiles of 2048 pairs: the tile scan's chunks meet, groups span them
    n = 2 * 4096 * 2048 + 12_345
    gen = torch.Generator().manual_seed(17)
    s = _scores(kind, n, gen)
    lab = torch.bernoulli(torch.full((n,), 0.3), generator=gen)
    xs, y, w, groups = _ext.calib_groups(s.cuda(), lab.cuda())
    g = int(groups[0])
    wx, wy, ww = _groups_oracle(s.numpy(), lab.numpy())
    assert g == wx.size
    assert np.array_equal(xs[:g].cpu().numpy(), wx)
    assert np.array_equal(y[:g].cpu().numpy(), wy)
    assert np.array_equal(w[:g].cpu().numpy(), ww)
