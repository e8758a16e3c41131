"""Writes tests/golden/golden.npz: seeded inputs with the outputs of the reference's OWN CPU
implementation of the path (torchisotonic 0.2.1, imported from a checkout of it), so that the
oracle and the CUDA kernels are pinned against the reference without it being present.

    python tests/golden/make_golden.py /path/to/torchisotonic

The reference JIT-builds its CPU op (src/torchisotonic/_ext.py:53-67) on first use. Cases follow
the reference's own tests: the batch x n grid and patterns of tests/test_cuda.py:31-134, NaN rows
(tests/test_isotonic.py:120-124), dtypes (test_isotonic.py:127-140), known-answer gradients
(tests/test_grad.py:32-56) and cancelling sums (tests/test_cuda.py:243-265). Each case stores
y, w (if any), the keyword arguments, the fit, the block starts (from the reference's _solve
with with_starts=True, _api.py:118-134) and, for gradient cases, the upstream gradient c and
d(sum(fit * c))/dy, /dw. bfloat16 arrays are stored as their uint16 bit patterns.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden.npz"


def pattern(name: str, n: int, g: torch.Generator) -> torch.Tensor:
    """The adversarial rows of the reference's tests/test_cuda.py:108-122."""
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
    return (i - n / 3) ** 2  # valley


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.bool:
        return t.numpy().astype(np.uint8)
    return t.numpy()


def main(ref_src: str) -> None:
    sys.path.insert(0, str(Path(ref_src) / "src"))
    import torchisotonic
    from torchisotonic import _api

    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    def add(name: str, y: torch.Tensor, w: torch.Tensor | None = None, grad: bool = False,
            c_seed: int = 0, **kw) -> None:
        assert name not in meta
        want = torchisotonic.isotonic(y, w, **kw)
        arrays[f"{name}/y"] = to_np(y)
        arrays[f"{name}/out"] = to_np(want)
        if w is not None:
            arrays[f"{name}/w"] = to_np(w)
        # where the blocks start (of the row-major [batch, n] problem along dim)
        dim = kw.get("dim", -1)
        out_dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
        acc = torch.float64 if out_dtype == torch.float64 else torch.float32
        rows = y.movedim(dim, -1)
        if rows.numel():
            flat_y = rows.reshape(-1, rows.shape[-1]).to(acc)
            flat_w = None
            if w is not None:
                flat_w = w.to(acc).broadcast_to(y.shape).movedim(dim, -1).reshape(flat_y.shape)
            _, starts = _api._solve(flat_y, flat_w, kw.get("increasing", True), True, True)
            arrays[f"{name}/starts"] = to_np(starts)
        if grad:
            gen = torch.Generator().manual_seed(c_seed)
            c = torch.randn(y.shape, generator=gen, dtype=torch.float64).to(y.dtype)
            yy = y.clone().requires_grad_()
            inputs = [yy]
            ww = None
            if w is not None:
                ww = w.clone().requires_grad_()
                inputs.append(ww)
            loss = (torchisotonic.isotonic(yy, ww, **kw) * c).sum()
            grads = torch.autograd.grad(loss, inputs)
            arrays[f"{name}/c"] = to_np(c)
            arrays[f"{name}/gy"] = to_np(grads[0])
            if w is not None:
                arrays[f"{name}/gw"] = to_np(grads[1])
        meta[name] = {
            "dtype": str(y.dtype).replace("torch.", ""),
            "weighted": w is not None,
            "grad": grad,
            "kwargs": kw,
        }

    # known answers (test_isotonic.py:127-140, test_grad.py:32-37, ties pool)
    for dt in (torch.float16, torch.bfloat16, torch.float32, torch.float64):
        add(f"known_{str(dt)[6:]}", torch.tensor([3.0, 1.0, 2.0, 5.0], dtype=dt))
    add("ties", torch.tensor([[1.0, 2.0, 2.0, 3.0]], dtype=torch.float64))
    add("single", torch.tensor([4.0]))
    add("block_average", torch.tensor([3.0, 1.0, 2.0]), grad=True, c_seed=1)
    add("nan_rows", torch.tensor([[3.0, math.nan, 2.0], [3.0, 1.0, 2.0]], dtype=torch.float64))

    # the batch x n grid of test_cuda.py:31-40
    for batch in (1, 3, 7):
        for n in (1, 2, 7, 100, 1000):
            if batch * n > 3000:
                continue
            for dt in (torch.float32, torch.float64):
                g = torch.Generator().manual_seed(batch * 1000 + n)
                y = torch.linspace(0, 3, n, dtype=dt) + torch.randn(batch, n, generator=g, dtype=dt)
                w = torch.rand(batch, n, generator=g, dtype=dt) + 0.1
                tag = f"grid_{batch}x{n}_{str(dt)[6:]}"
                add(f"{tag}_plain", y)
                add(f"{tag}_w", y, w)
                add(f"{tag}_dec_clip", y, w, increasing=False, y_min=-0.5, y_max=2.0)

    # patterns of test_cuda.py:105-134
    for name in ("increasing", "decreasing", "saw", "cliff", "walk", "constant", "valley"):
        for n in (700, 1025, 2100):
            g = torch.Generator().manual_seed(n)
            y = pattern(name, n, g)[None]
            w = torch.rand(1, n, generator=g, dtype=torch.float64) + 0.1
            add(f"pat_{name}_{n}_f64", y)
            add(f"pat_{name}_{n}_f64_w", y, w)
            add(f"pat_{name}_{n}_f64_w_dec", y, w, increasing=False)
            add(f"pat_{name}_{n}_f32", y.float())

    # NaN rows in a batch (test_cuda.py:51-55)
    g = torch.Generator().manual_seed(5)
    y = torch.randn(30, 50, generator=g, dtype=torch.float64)
    y[7, 3] = math.nan
    y[29, 49] = math.nan
    add("nan_batch", y)
    w = torch.rand(30, 50, generator=g, dtype=torch.float64) + 0.1
    add("nan_batch_grad", y, w, grad=True, c_seed=2)

    # other dims and low precision (test_cuda.py:58-62)
    g = torch.Generator().manual_seed(6)
    y = torch.randn(4, 60, 5, generator=g)
    add("dim1_f32", y, dim=1)
    add("dim1_f16", y.half(), dim=1)
    add("dim1_bf16", y.bfloat16(), dim=1)
    add("dim0_f64_w", y.double(), torch.rand(4, 60, 5, generator=g, dtype=torch.float64) + 0.1,
        dim=0)
    add("int_input", torch.tensor([3, 1, 2]))
    add("broadcast_w", torch.tensor([[3.0, 1.0, 2.0], [1.0, 3.0, 2.0]], dtype=torch.float64),
        torch.tensor([1.0, 2.0, 3.0], dtype=torch.float64))

    # gradients (test_grad.py and test_cuda.py:137-157), clipped and decreasing too
    for (batch, n) in ((5, 31), (9, 64), (2, 1000), (1, 2100)):
        for dt in (torch.float32, torch.float64):
            g = torch.Generator().manual_seed(n)
            y = torch.linspace(0, 3, n, dtype=dt) + torch.randn(batch, n, generator=g, dtype=dt)
            w = torch.rand(batch, n, generator=g, dtype=dt) + 0.1
            tag = f"grad_{batch}x{n}_{str(dt)[6:]}"
            add(f"{tag}_w_dec", y, w, grad=True, c_seed=n, increasing=False)
            add(f"{tag}_plain", y, grad=True, c_seed=n + 1)
            add(f"{tag}_w_clip", y, w, grad=True, c_seed=n + 2, y_min=0.5, y_max=2.5)
    g = torch.Generator().manual_seed(7)
    yb = (torch.cumsum(0.1 + torch.randn(16, 64, generator=g), 1)
          + 0.3 * torch.randn(16, 64, generator=g)).bfloat16()
    wb = 0.1 + torch.rand(16, 64, generator=g)
    add("grad_bf16_quantile", yb, wb, grad=True, c_seed=8)

    # close values: increasing rows, their own fit (test_grad.py:40-56)
    one = torch.tensor(1.0).view(torch.int32)
    add("consecutive_f32", (one + torch.arange(1000, dtype=torch.int32)).view(torch.float32)[None],
        grad=True, c_seed=9)

    # cancelling sums (test_cuda.py:243-265), float64
    for n in (500, 3000):
        for big in (1e3, 1e6):
            g = torch.Generator().manual_seed(n)
            k = torch.arange(n) % 64
            y = torch.where(k < 32, big, 1.0).double()
            y[k == 32] = -32 * big
            y += 1e-3 * (-1.0) ** k * (k > 32) + 1e-6 * torch.randn(n, generator=g, dtype=torch.float64)
            add(f"cancel_{n}_{int(big)}", y[None])

    # empty inputs (test_isotonic.py:143-146)
    add("empty_3x0", torch.empty(3, 0))

    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {len(meta)} cases to {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/torchisotonic-checkout")
    main(sys.argv[1])
