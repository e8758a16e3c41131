"""The oracle is pinned before it is trusted: against the fixtures the reference's own CPU
implementation wrote (tests/golden/make_golden.py) and against the reference's solver compiled
here (oracle/_ref). CPU only."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_case, golden_names
from golden_util import DTYPES, out_tensor, tensor

import oracle

FIT_CASES = golden_names(lambda k, m: "out" in m or True)


def _inputs(case: dict) -> tuple[torch.Tensor, torch.Tensor | None, dict]:
    y = tensor(case["y"], case["dtype"])
    w = tensor(case["w"], "float64" if case["dtype"] == "float64" else "float32") \
        if "w" in case else None
    if w is not None and case["dtype"] in ("float32", "float64"):
        w = w.to(DTYPES[case["dtype"]])
    return y, w, dict(case["kwargs"])


@pytest.mark.parametrize("name", FIT_CASES)
def test_reference_precision_is_bit_exact(name: str) -> None:
    # The restatement, in the reference's own precision and operation order, reproduces the
    # reference CPU op bit for bit: values and block starts.
    case = golden_case(name)
    y, w, kw = _inputs(case)
    got, starts = oracle.isotonic(y, w, precision=oracle.PREC_REFERENCE, with_starts=True, **kw)
    want = out_tensor(case)
    assert got.dtype == want.dtype and got.shape == want.shape
    assert torch.equal(got.reshape(-1).isnan(), want.reshape(-1).isnan())
    if got.dtype in (torch.bfloat16, torch.float16):
        assert torch.equal(got.float().nan_to_num(), want.float().nan_to_num())
    else:
        assert torch.equal(got.nan_to_num(), want.nan_to_num())
    if "starts" in case:
        assert np.array_equal(starts.numpy().astype(np.uint8), case["starts"])


@pytest.mark.parametrize("name", FIT_CASES)
def test_extended_precision_matches_reference(name: str) -> None:
    # The exact-partition oracle agrees with the reference within the reference's own test
    # tolerances (tests/test_cuda.py:27: 1e-12 for float64, 1e-4 for float32, 1e-2 half), and
    # on float64 data also in the block partition.
    case = golden_case(name)
    y, w, kw = _inputs(case)
    got, starts = oracle.isotonic(y, w, precision=oracle.PREC_EXTENDED, with_starts=True, **kw)
    want = out_tensor(case)
    tol = {"float64": 1e-12, "float32": 1e-4}.get(case["dtype"], 1e-2)
    if case["dtype"] == "float64":
        scale = max(1.0, float(y.double().nan_to_num().abs().max())) if y.numel() else 1.0
        torch.testing.assert_close(got, want, rtol=tol, atol=tol * scale, equal_nan=True)
    else:
        torch.testing.assert_close(got.double(), want.double(), rtol=tol, atol=tol, equal_nan=True)
    if "starts" in case and case["dtype"] == "float64" and not name.startswith("cancel"):
        assert np.array_equal(starts.numpy().astype(np.uint8), case["starts"])


@pytest.mark.parametrize("name", golden_names(lambda k, m: m["grad"]))
def test_gradient_oracle_matches_reference(name: str) -> None:
    # The backward restatement (block sums of the clamp-masked upstream gradient) against the
    # reference's autograd on its CPU op.
    case = golden_case(name)
    y, w, kw = _inputs(case)
    acc = torch.float64 if y.dtype == torch.float64 else torch.float32
    kw.pop("dim", None)
    increasing = kw.pop("increasing", True)
    y_min, y_max = kw.pop("y_min", None), kw.pop("y_max", None)
    flat_y = y.to(acc).reshape(-1, y.shape[-1]).numpy()
    flat_w = None if w is None else w.to(acc).reshape(flat_y.shape).numpy()
    fit, starts = oracle.fit(flat_y, flat_w, increasing=increasing, precision=oracle.PREC_EXTENDED)
    c = tensor(case["c"], case["dtype"]).to(acc).reshape(flat_y.shape).numpy()
    gy, gw = oracle.grad(fit, starts, c, flat_w, flat_y if w is not None else None,
                         y_min=y_min, y_max=y_max)
    tol = 1e-9 if acc == torch.float64 else 1e-4
    want_gy = tensor(case["gy"], case["dtype"]).double().reshape(gy.shape).numpy()
    if case["dtype"] == "bfloat16":
        gy = torch.from_numpy(gy).bfloat16().double().numpy()
        tol = 1e-2
    np.testing.assert_allclose(gy, want_gy, rtol=tol, atol=tol)
    if w is not None:
        want_gw = tensor(case["gw"], "float64" if acc == torch.float64 else "float32")
        scale = 1 + float(np.nan_to_num(np.abs(flat_y)).max())
        np.testing.assert_allclose(gw, want_gw.double().reshape(gw.shape).numpy(),
                                   rtol=tol, atol=tol * scale)


@pytest.mark.skipif(oracle.ref_lib() is None, reason="reference solver not built here")
@pytest.mark.parametrize("name", golden_names(lambda k, m: m["dtype"] in ("float32", "float64")
                                              and "y_min" not in m["kwargs"]
                                              and "dim" not in m["kwargs"]))
def test_reference_solver_build_matches_fixtures(name: str) -> None:
    # The reference's own pava.h compiled here reproduces the fixtures bit for bit, so it can
    # stand for the reference as the CPU baseline.
    case = golden_case(name)
    y, w, kw = _inputs(case)
    if y.numel() == 0:
        return
    flat_y = y.reshape(-1, y.shape[-1]).contiguous().numpy()
    flat_w = None if w is None else w.broadcast_to(y.shape).reshape(flat_y.shape).contiguous().numpy()
    out, starts = oracle.ref_fit(flat_y, flat_w, increasing=kw.get("increasing", True))
    want = case["out"].reshape(out.shape)
    np.testing.assert_array_equal(np.isnan(out), np.isnan(want))
    np.testing.assert_array_equal(np.nan_to_num(out), np.nan_to_num(want))
    if "starts" in case:
        np.testing.assert_array_equal(starts.astype(np.uint8), case["starts"])


def test_known_answers() -> None:
    # [3, 1, 2, 5] -> [2, 2, 2, 5] (test_isotonic.py:127-134); ties pool: [1, 2, 2, 3] has
    # blocks starting at 0, 1, 3; a NaN makes its row NaN with one block at 0 (pava.h:30-37).
    out, st = oracle.fit(np.array([[3.0, 1.0, 2.0, 5.0]]))
    assert out.tolist() == [[2.0, 2.0, 2.0, 5.0]] and st.tolist() == [[True, False, False, True]]
    out, st = oracle.fit(np.array([[1.0, 2.0, 2.0, 3.0]]))
    assert st.tolist() == [[True, True, False, True]]
    out, st = oracle.fit(np.array([[3.0, np.nan, 2.0]], dtype=np.float32))
    assert np.isnan(out).all() and st.tolist() == [[True, False, False]]
    out, _ = oracle.fit(np.array([[1.0, 2.0, 3.0]]), increasing=False)
    assert out.tolist() == [[2.0, 2.0, 2.0]]
    gy, _ = oracle.grad(np.full((1, 3), 2.0), np.array([[True, False, False]]),
                        np.array([[1.0, 2.0, 6.0]]))
    assert gy.tolist() == [[3.0, 3.0, 3.0]]  # test_grad.py:32-37


def test_extended_precision_resolves_float32_ties() -> None:
    # Means that float32 sums cannot tell apart: (1 + u, 1, 1) blocks with u the float32
    # spacing at 1 have means 1 + u / 3 > 1; the extended oracle keeps them apart from a
    # following block of 1 + u / 2 > 1 + u / 3, as the exact problem does.
    u = np.float32(np.finfo(np.float32).eps)
    y = np.array([[1 + u, 1, 1, 1 + u, 1]], dtype=np.float32)
    _, st = oracle.fit(y, precision=oracle.PREC_EXTENDED)
    assert st.tolist() == [[True, False, False, True, False]]
