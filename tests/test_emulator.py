"""The tile kernel's phase logic (fit_core.cuh, compiled for the host by tests/emu) against the
oracle, on CPU: thread-level PAVA, the merge rounds' bookkeeping and the expand, for every
segment width from one thread per row to 256 threads per row."""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle

EMU = Path(__file__).resolve().parent / "emu"


def _lib() -> ctypes.CDLL:
    src = EMU / "emu_fit.cpp"
    so = EMU / "libemu.so"
    deps = [src, *(EMU.parent.parent / "torchisotonic_b200" / "csrc").glob("*.cuh")]
    if not so.exists() or any(p.stat().st_mtime > so.stat().st_mtime for p in deps):
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", str(so), str(src)],
                       check=True)
    lib = ctypes.CDLL(str(so))
    p, i64, i = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.emu_fit_rows.argtypes = [p, p, p, p, i64, i, i, i]
    lib.emu_fastdiv.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    lib.emu_fastdiv.restype = ctypes.c_uint32
    return lib


LIB = _lib()


def emu(y: np.ndarray, w: np.ndarray | None, increasing: bool = True, exact: bool = True):
    y = np.ascontiguousarray(y, dtype=np.float64)
    wc = None if w is None else np.ascontiguousarray(w, dtype=np.float64)
    out = np.empty_like(y)
    st = np.empty(y.shape, dtype=np.uint8)
    rc = LIB.emu_fit_rows(y.ctypes.data, None if wc is None else wc.ctypes.data, out.ctypes.data,
                          st.ctypes.data, y.shape[0], y.shape[1], int(increasing), int(exact))
    assert rc == 0
    return out, st.astype(bool)


def pattern(name: str, n: int, rng: np.random.Generator) -> np.ndarray:
    i = np.arange(n, dtype=np.float64)
    return {
        "increasing": i,
        "decreasing": -i,
        "saw": i % 7 + (i % 1500) * 0.1,
        "cliff": np.where(i == n - 1, -1e9, i),
        "walk": rng.standard_normal(n).cumsum(),
        "constant": np.ones(n),
        "valley": (i - n / 3) ** 2,
        "noise": 0.001 * i + rng.standard_normal(n),
        "steps": np.floor(i / 5) - (i % 5 == 0) * 3.0,
    }[name]


NS = [1, 2, 3, 15, 16, 17, 31, 32, 33, 64, 100, 255, 256, 257, 511, 512, 513, 1000, 1023, 1024,
      1025, 2048, 2049, 3000, 4095, 4096]


@pytest.mark.parametrize("n", NS)
@pytest.mark.parametrize("weighted", [False, True])
def test_random_rows(n: int, weighted: bool) -> None:
    rng = np.random.default_rng(n)
    batch = max(1, min(40, 8192 // n))
    y = (np.linspace(0, 3, n) + rng.standard_normal((batch, n))).astype(np.float32).astype(np.float64)
    w = (rng.random((batch, n)) + 0.1).astype(np.float32).astype(np.float64) if weighted else None
    for inc in (True, False):
        out, st = emu(y, w, inc)
        want, wst = oracle.fit(y.astype(np.float32), None if w is None else w.astype(np.float32),
                               increasing=inc)
        np.testing.assert_array_equal(st, wst)
        np.testing.assert_allclose(out.astype(np.float32), want, rtol=2e-7, atol=1e-6)


@pytest.mark.parametrize("name", ["increasing", "decreasing", "saw", "cliff", "walk", "constant",
                                  "valley", "noise", "steps"])
@pytest.mark.parametrize("n", [7, 33, 700, 1025, 4096])
def test_patterns(name: str, n: int) -> None:
    rng = np.random.default_rng(n)
    y = np.stack([pattern(name, n, rng) for _ in range(3)])
    # float32-representable weights: w y is then exact in double, so exact ties (the steps and
    # constant patterns) are ties for the kernels too. With arbitrary float64 weights w y rounds,
    # and ties closer than that rounding are decided by it - as in the reference's double path.
    w = (rng.random(y.shape) + 0.1).astype(np.float32).astype(np.float64)
    for ww in (None, w):
        for inc in (True, False):
            out, st = emu(y, ww, inc)
            want, wst = oracle.fit(y, ww, increasing=inc)
            np.testing.assert_array_equal(st, wst)
            scale = max(1.0, float(np.abs(y).max()))
            np.testing.assert_allclose(out, want, rtol=1e-12, atol=1e-12 * scale)


def test_nan_rows() -> None:
    rng = np.random.default_rng(3)
    y = rng.standard_normal((20, 300))
    y[3, 7] = np.nan
    y[19, 299] = np.nan
    out, st = emu(y, None)
    want, wst = oracle.fit(y)
    np.testing.assert_array_equal(np.isnan(out), np.isnan(want))
    np.testing.assert_array_equal(st, wst)


def test_fast_mode_band() -> None:
    rng = np.random.default_rng(4)
    y = (np.linspace(0, 3, 500) + rng.standard_normal((10, 500))).astype(np.float32)
    out, _ = emu(y.astype(np.float64), None, exact=False)
    want, _ = oracle.fit(y)
    np.testing.assert_allclose(out, want, rtol=1e-3, atol=1e-3)


def test_fastdiv() -> None:
    rng = np.random.default_rng(5)
    for d in [1, 2, 3, 5, 7, 16, 17, 100, 1000, 4096, 5000, 65535, 2**20 + 7, 2**30 + 3]:
        for n in list(rng.integers(0, 2**31 - 1, 2000)) + [0, d - 1, d, d + 1, 2**31 - 2]:
            assert LIB.emu_fastdiv(int(n), d) == int(n) // d


@pytest.mark.parametrize("name", ["collinear", "offset", "consecutive"])
def test_float32_near_collinear_partition(name: str) -> None:
    # float32 data around a large value (tests/test_cuda.py:224-240): exact ties everywhere.
    # Fitting w (y - y0) keeps the double sums exact, so the partition is the exact one.
    n = 1000
    rng = np.random.default_rng(n)
    i = np.arange(n, dtype=np.float64)
    one = np.float32(1.0).view(np.int32)
    y = {
        "collinear": 1e6 + 1e-3 * i + 1e-9 * rng.standard_normal(n),
        "offset": 1e6 + rng.standard_normal(n),
        "consecutive": (one + np.arange(n, dtype=np.int32)).view(np.float32).astype(np.float64),
    }[name].astype(np.float32)
    u = rng.random(n).astype(np.float32)
    for w in (None, u + np.float32(0.1), np.exp(8 * u).astype(np.float32)):
        yy = y[None].astype(np.float64)
        ww = None if w is None else w[None].astype(np.float64)
        out, st = emu(yy, ww)
        want, wst = oracle.fit(y[None], None if w is None else w[None])
        np.testing.assert_array_equal(st, wst)
        assert (np.diff(out.astype(np.float32)[0]) >= 0).all()
