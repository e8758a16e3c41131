"""Soft rank on the fit (the reference's in-model consumer, paper/soft_rank.py:31-55).

CPU: the numpy oracle pinned to fixtures made by the reference's own fit inside that
composition (tests/golden/make_soft_rank_golden.py): float64 within 1e-12 of the scale, values
and gradients; float32 bit-exact in the reference's precision. GPU: soft_rank and its gradient
against the fixtures (float64) and against the extended-precision oracle (float32: the
kernels' pooling decisions are exact, like the oracle's, so within a few units in the last
place of the ranks' scale), gradcheck in float64, and properties at larger sizes: the ranks of
a row sum to n (n + 1) / 2, hard ranks for a small strength, order kept.
"""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import torchisotonic_b200

FIX = Path(__file__).resolve().parent / "golden" / "soft_rank.npz"


@lru_cache(maxsize=1)
def fixtures() -> dict[str, dict]:
    z = np.load(FIX)
    meta = json.loads(bytes(z["__meta__"]).decode())
    return {name: {"strength": m["strength"],
                   **{k: z[f"{name}/{k}"] for k in ("x", "c", "out", "grad")}}
            for name, m in meta.items()}


NAMES = sorted(fixtures())


def _close(got: np.ndarray, want: np.ndarray, rel: float) -> None:
    scale = max(1.0, float(np.abs(want).max()))
    np.testing.assert_allclose(got, want, rtol=0, atol=rel * scale)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_composition(name: str) -> None:
    c = fixtures()[name]
    if c["x"].dtype == np.float64:
        out, grad = oracle.soft_rank(c["x"], c["strength"], c["c"])
        _close(out, c["out"], 1e-12)
        _close(grad, c["grad"], 1e-12)
    else:
        out, grad = oracle.soft_rank(c["x"], c["strength"], c["c"],
                                     precision=oracle.PREC_REFERENCE)
        assert np.array_equal(out, c["out"])
        _close(grad, c["grad"], 1e-6)


def test_soft_rank_argument_checks() -> None:
    with pytest.raises(TypeError):
        torchisotonic_b200.soft_rank([1.0, 2.0])  # type: ignore[arg-type]
    with pytest.raises(TypeError, match="float32 or float64"):
        torchisotonic_b200.soft_rank(torch.zeros(2, 3, dtype=torch.int64))
    with pytest.raises(ValueError, match="> 0"):
        torchisotonic_b200.soft_rank(torch.zeros(2, 3), 0.0)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torchisotonic_b200.soft_rank(torch.zeros(2, 3))


def _run(x: np.ndarray, strength: float, c: np.ndarray):
    xt = torch.from_numpy(x).cuda().requires_grad_()
    out = torchisotonic_b200.soft_rank(xt, strength)
    (g,) = torch.autograd.grad(out, xt, torch.from_numpy(c).cuda())
    return out.detach().cpu().numpy(), g.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_soft_rank_matches_reference(name: str) -> None:
    c = fixtures()[name]
    out, grad = _run(c["x"], c["strength"], c["c"])
    if c["x"].dtype == np.float64:
        _close(out, c["out"], 1e-12)
        _close(grad, c["grad"], 1e-12)
    else:
        want, want_g = oracle.soft_rank(c["x"], c["strength"], c["c"])
        _close(out, want, 4 * 2.0**-24)
        _close(grad, want_g, 1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1024, 100), (64, 10_000), (2, 300_000)])
@pytest.mark.parametrize("strength", [1.0, 1e-3])
def test_soft_rank_properties(shape: tuple[int, int], strength: float) -> None:
    gen = torch.Generator(device="cuda").manual_seed(shape[1])
    x = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float64)
    r = torchisotonic_b200.soft_rank(x, strength)
    n = shape[1]
    torch.testing.assert_close(r.sum(-1), torch.full((shape[0],), n * (n + 1) / 2,
                                                     dtype=torch.float64, device="cuda"),
                               rtol=1e-12, atol=0)
    order = torch.argsort(x, dim=-1)
    ranked = r.gather(-1, order)
    assert bool((ranked[:, 1:] >= ranked[:, :-1] - 1e-9 * n).all())  # order kept
    # distinct values at least `strength` x 2 apart: the hard ranks, exactly
    p = torch.argsort(torch.rand(shape, generator=gen, device="cuda"), dim=-1).double()
    hard = torchisotonic_b200.soft_rank(p * (2 * strength), strength)
    torch.testing.assert_close(hard, p + 1, rtol=0, atol=1e-12 * n)


@pytest.mark.gpu
def test_soft_rank_gradcheck() -> None:
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(3, 9, generator=gen, device="cuda", dtype=torch.float64).requires_grad_()
    assert torch.autograd.gradcheck(lambda t: torchisotonic_b200.soft_rank(t, 0.7), (x,))


@pytest.mark.gpu
def test_soft_rank_leading_dims() -> None:
    x = torch.randn(2, 3, 50, device="cuda")
    r = torchisotonic_b200.soft_rank(x, 0.5)
    assert r.shape == x.shape
    torch.testing.assert_close(r.reshape(6, 50), torchisotonic_b200.soft_rank(x.reshape(6, 50),
                                                                              0.5))
