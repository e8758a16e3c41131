"""The operator layer on the GPU: the torch.library operators (torchisotonic_b200/ops.py) under
torch.library.opcheck and torch.compile(fullgraph=True), and the reference-side binding that
INTEGRATION.md documents - its code block executed as written - driven the way the reference's
own _api.py drives its operators (src/torchisotonic/_api.py:43-97: cast, the operator with block
starts, clamp; the backward through isotonic_grad(out, starts, g, w, y)), against the golden
fixtures the reference wrote."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import golden_case, golden_names
from golden_util import tensor

import torchisotonic_b200
from torchisotonic_b200 import _ext, ops

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _binding() -> dict:
    """The INTEGRATION.md binding (its first Python code block), loading this library."""
    text = (ROOT / "INTEGRATION.md").read_text()
    block = re.search(r"## The binding \(Python, ctypes\)\s*```python\n(.*?)```", text, re.S)
    assert block, "INTEGRATION.md has no binding code block"
    code = block.group(1).replace("/path/to/libtiso.so", str(_ext.LIB_PATH))
    ns: dict = {}
    exec(compile(code, "INTEGRATION.md", "exec"), ns)  # noqa: S102 - the documented binding
    return ns


def _eligible(name: str, meta: dict) -> bool:
    return (meta["dtype"] in ("float32", "float64") and "dim" not in meta["kwargs"]
            and not name.startswith("empty"))


@pytest.mark.parametrize("name", golden_names(_eligible))
def test_integration_binding_against_golden(name: str) -> None:
    b = _binding()
    case = golden_case(name)
    kw = case["kwargs"]
    y = tensor(case["y"], case["dtype"])
    n = y.shape[-1]
    flat_y = y.reshape(-1, n).cuda()
    flat_w = None
    if "w" in case:
        flat_w = torch.from_numpy(np.array(case["w"])).to(y.dtype).broadcast_to(y.shape)
        flat_w = flat_w.reshape(-1, n).contiguous().cuda()
    y_min, y_max = kw.get("y_min"), kw.get("y_max")
    yg = flat_y.clone().requires_grad_(case["grad"])
    wg = None if flat_w is None else flat_w.clone().requires_grad_(case["grad"])
    out, starts = b["isotonic_tiles"](yg.detach(), None if wg is None else wg.detach(),
                                       kw.get("increasing", True), True, True)
    clipped = out if (y_min is None and y_max is None) else out.clamp(min=y_min, max=y_max)
    want = torch.from_numpy(np.array(case["out"])).reshape(flat_y.shape)
    tol = 1e-12 if y.dtype == torch.float64 else 1e-4
    sc = max(1.0, float(y.double().nan_to_num(0).abs().max())) if y.numel() else 1.0
    torch.testing.assert_close(clipped.cpu().double(), want.double(), rtol=tol,
                               atol=tol * (sc if y.dtype == torch.float64 else 1.0),
                               equal_nan=True)
    if "starts" in case and not torch.isnan(flat_y).any():
        assert torch.equal(starts.cpu(), torch.from_numpy(np.array(case["starts"])).reshape(
            flat_y.shape).bool())
    if case["grad"]:
        c = torch.from_numpy(np.array(case["c"])).to(y.dtype).reshape(flat_y.shape).cuda()
        # the clamp's backward (inclusive bounds), then the operator's
        g = c
        if y_min is not None or y_max is not None:
            lo = -np.inf if y_min is None else y_min
            hi = np.inf if y_max is None else y_max
            g = c * ((out >= lo) & (out <= hi))
        gy, gw = b["isotonic_grad"](out, starts, g.contiguous(), flat_w,
                                     flat_y if flat_w is not None else None)
        gtol = 1e-9 if y.dtype == torch.float64 else 2e-5
        torch.testing.assert_close(gy.cpu(), torch.from_numpy(np.array(case["gy"])).reshape(
            flat_y.shape).to(y.dtype), rtol=gtol, atol=gtol, equal_nan=True)
        if flat_w is not None and "gw" in case:
            torch.testing.assert_close(gw.cpu(), torch.from_numpy(np.array(case["gw"])).reshape(
                flat_y.shape).to(y.dtype), rtol=gtol, atol=gtol * 10, equal_nan=True)


def _inputs(dtype=torch.float32, b=37, n=300, seed=0):
    g = torch.Generator().manual_seed(seed)
    y = (torch.linspace(0, 3, n) + torch.randn(b, n, generator=g)).to(dtype).cuda()
    w = (torch.rand(b, n, generator=g) + 0.1).to(_ext.acc_dtype(dtype)).cuda()
    return y, w


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
def test_opcheck(dtype) -> None:
    y, w = _inputs(dtype)
    y.requires_grad_()
    w.requires_grad_()
    torch.library.opcheck(ops.fit, (y, w, True, True, True, 0.5, 2.5))
    torch.library.opcheck(ops.fit, (y.detach(), None, False, True, False, None, None))
    _, st = ops.fit(y.detach(), w.detach(), True, True, True, None, None)
    g = torch.randn_like(y.detach())
    torch.library.opcheck(ops.fit_grad, (st, g, w.detach(), y.detach(), True, True, None, 2.0))
    if dtype != torch.bfloat16:
        torch.library.opcheck(ops.isotonic_tiles, (y.detach(), w.detach(), True, True, True))
        out, st2 = ops.isotonic_tiles(y.detach(), w.detach(), True)
        torch.library.opcheck(ops.isotonic_grad, (out, st, g, w.detach(), y.detach()))


def test_reference_schema_operators_match_the_fused_path() -> None:
    y, w = _inputs(torch.float64)
    out, st = torch.ops.torchisotonic_b200.isotonic_tiles(y, w, False, True, True)
    want = torchisotonic_b200.isotonic(y, w, increasing=False)
    assert torch.equal(out, want)
    g = torch.randn_like(y)
    gy, gw = torch.ops.torchisotonic_b200.isotonic_grad(out, st, g, w, y)
    yy, ww = y.clone().requires_grad_(), w.clone().requires_grad_()
    ey, ew = torch.autograd.grad((torchisotonic_b200.isotonic(yy, ww, increasing=False) * g).sum(),
                                 (yy, ww))
    torch.testing.assert_close(gy, ey, rtol=0, atol=0)
    torch.testing.assert_close(gw, ew, rtol=0, atol=0)
    gy2, gw2 = torch.ops.torchisotonic_b200.isotonic_grad(out, st, g, w, None)
    assert gw2.numel() == 0 and torch.equal(gy2, gy)


def test_compile_fullgraph_forward_and_backward() -> None:
    torch._dynamo.reset()
    y, w = _inputs(torch.float32)

    def f(y, w):
        return (torchisotonic_b200.isotonic(y, w, y_min=0.5, y_max=2.5) ** 2).sum()

    cf = torch.compile(f, fullgraph=True)
    ye, we = y.clone().requires_grad_(), w.clone().requires_grad_()
    yc, wc = y.clone().requires_grad_(), w.clone().requires_grad_()
    le = f(ye, we)
    le.backward()
    lc = cf(yc, wc)
    lc.backward()
    torch.testing.assert_close(lc, le, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(yc.grad, ye.grad, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(wc.grad, we.grad, rtol=1e-6, atol=1e-6)
    with torch.no_grad():
        torch.testing.assert_close(torch.compile(lambda y: torchisotonic_b200.isotonic(
            y, increasing=False), fullgraph=True)(y), torchisotonic_b200.isotonic(y, increasing=False))


def test_non_positive_weight_raises_through_the_operator() -> None:
    y, w = _inputs(torch.float32)
    w[3, 7] = 0.0
    with pytest.raises(ValueError, match="strictly positive"):
        torchisotonic_b200.isotonic(y, w)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_check_weights_through_the_c_abi(dtype) -> None:
    # tiso_check_weights: the flag set for any weight not > 0 (NaN included), unaligned starts
    # and tails read element by element
    so = _ext.lib()
    flag = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    code = _ext._DTYPES[dtype]
    for n in (1, 3, 1000, 1_000_003):
        w = torch.rand(n + 1, dtype=dtype, device="cuda") + 0.1
        for off in (0, 1):  # an aligned and an unaligned start
            v = w[off:off + n]
            assert so.tiso_check_weights(code, v.data_ptr(), n, flag.data_ptr(), stream) == 0
            assert int(flag.item()) == 0
            for bad in (0.0, -1.0, float("nan")):
                u = v.clone()
                u[n // 2] = bad
                assert so.tiso_check_weights(code, u.data_ptr(), n, flag.data_ptr(), stream) == 0
                assert int(flag.item()) == 1
    assert so.tiso_check_weights(code, None, 0, flag.data_ptr(), stream) == 0
    assert int(flag.item()) == 0


def test_non_positive_weight_raises_for_large_weights() -> None:
    # weights past the early check's size: the fit's own fused check raises the same error
    y = torch.randn(2048, 8200, device="cuda")
    w = torch.rand(2048, 8200, device="cuda") + 0.1
    assert w.numel() * 4 > _ext.WeightCheck.EARLY_CHECK_BYTES
    torchisotonic_b200.isotonic(y, w)
    w[1000, 4000] = 0.0
    with pytest.raises(ValueError, match="strictly positive"):
        torchisotonic_b200.isotonic(y, w)


def test_weight_checks_reuse_their_flags() -> None:
    # the check's flag, pinned word and event are reused per thread and device: bad and good
    # weights in turn, at a size checked by its own pass and at one checked inside the fit, and
    # from a second thread, each call seeing only its own weights
    import threading

    for shape in ((64, 300), (2048, 8200)):
        y = torch.randn(*shape, device="cuda")
        good = torch.rand(*shape, device="cuda") + 0.1
        bad = good.clone()
        bad[shape[0] // 2, 7] = -1.0
        for _ in range(3):
            with pytest.raises(ValueError, match="strictly positive"):
                torchisotonic_b200.isotonic(y, bad)
            torchisotonic_b200.isotonic(y, good)
        errors = []

        def worker() -> None:
            try:
                torchisotonic_b200.isotonic(y, good)
                try:
                    torchisotonic_b200.isotonic(y, bad)
                    errors.append("bad weights passed")
                except ValueError:
                    pass
            except Exception as e:  # noqa: BLE001 - reported below
                errors.append(repr(e))

        t = threading.Thread(target=worker)
        t.start()
        t.join()
        assert not errors, errors
