"""Differentiable ranking on the isotonic fit: the in-model consumer of the fit's forward and
backward that the reference benchmarks (paper/soft_rank.py:31-55, torchsort's ``SoftRank`` with
the l2 regularisation and torchisotonic as its solver).

``soft_rank(x, regularization_strength)`` is the projection of ``x / strength`` onto the
permutahedron of the ranks 1..n: sort each row descending, fit ``s - (n, n-1, ..., 1)`` with a
non-increasing isotonic regression, and put ``s - fit`` back in the input's order. Small
strengths give the hard ranks (1 for the smallest), large ones pull every rank to the mean. The
gradient is the projection's: ``scale (g - P^T A P g)``, A the fit's averaging over its blocks.
Here the fit and its backward run in this library's kernels (through the C ABI, with the block
starts kept from the forward), the sort is torch's.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from torchisotonic_b200 import _ext


class _SoftRank(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, x: Tensor, strength: float) -> Tensor:
        scale = 1.0 / strength
        # stable: tied values keep their order, so ties get the ranks the reference's
        # CPU composition gives them
        s, perm = torch.sort(x * scale, dim=-1, descending=True, stable=True)
        n = x.shape[-1]
        w = torch.arange(n, 0, -1, dtype=x.dtype, device=x.device)  # n, n-1, ..., 1
        z = (s - w).contiguous()
        dual, starts = _ext.isotonic_tiles(z, None, increasing=False, exact=True,
                                           with_starts=any(ctx.needs_input_grad))
        out = torch.empty_like(s).scatter_(-1, perm, s - dual)
        ctx.save_for_backward(perm, starts)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx: Any, g: Tensor) -> tuple[Tensor, None]:
        perm, starts = ctx.saved_tensors
        sorted_g = g.gather(-1, perm).contiguous()
        avg, _ = _ext.isotonic_grad(starts, sorted_g, None, None, True, False)
        grad = g - torch.empty_like(g).scatter_(-1, perm, avg)
        return grad * ctx.scale, None


def soft_rank(values: Tensor, regularization_strength: float = 1.0) -> Tensor:
    """Soft ranks of every row of ``values`` (a [batch, n] CUDA tensor, float32 or float64;
    leading dimensions are flattened and restored), with the l2 regularisation of torchsort's
    ``soft_rank`` (the reference's paper/soft_rank.py:31-55). Differentiable in ``values``."""
    if not isinstance(values, Tensor):
        raise TypeError(f"values must be a torch.Tensor, got {type(values).__name__}")
    if values.dim() < 1 or values.shape[-1] < 1:
        raise ValueError("values must have a last dimension of at least one element")
    if not values.dtype.is_floating_point or values.dtype in (torch.float16, torch.bfloat16):
        raise TypeError("values must be float32 or float64")
    if not regularization_strength > 0:
        raise ValueError("regularization_strength must be > 0")
    if not values.is_cuda:
        raise RuntimeError(
            "torchisotonic_b200 runs on CUDA tensors only (no CPU fallback); "
            "move values to a CUDA device"
        )
    shape = values.shape
    rows = values.reshape(-1, shape[-1])
    if rows.shape[0] == 0:
        return values.clone()
    out: Tensor = _SoftRank.apply(rows, float(regularization_strength))
    return out.reshape(shape)
