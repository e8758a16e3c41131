"""Writes tests/golden/soft_rank.npz: soft ranks and their gradients from the composition the
reference benchmarks as its in-model consumer (paper/soft_rank.py:31-55: sort descending,
non-increasing isotonic fit of s - (n..1), s - fit put back in order; backward
g - P^T A P g), run on the CPU with the reference's own fit and autograd (torchisotonic 0.2.1,
imported from a checkout of it).

    python tests/golden/make_soft_rank_golden.py /path/to/torchisotonic
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "soft_rank.npz"


def main(ref_src: str) -> None:
    sys.path.insert(0, str(Path(ref_src) / "src"))
    import torchisotonic

    def ranks(x: torch.Tensor, strength: float) -> torch.Tensor:
        scale = 1.0 / strength
        s, perm = torch.sort(x * scale, dim=-1, descending=True, stable=True)
        n = x.shape[-1]
        w = torch.arange(n, 0, -1, dtype=x.dtype)
        dual = torchisotonic.isotonic(s - w, increasing=False)
        return torch.empty_like(s).scatter(-1, perm, s - dual)

    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    g = torch.Generator().manual_seed(21)
    for dtype in (torch.float64, torch.float32):
        for b, n in ((16, 1), (8, 7), (4, 100), (2, 1000), (1, 5000)):
            for sname, strength in (("1", 1.0), ("1_over_n", 1.0 / n), ("10", 10.0)):
                name = f"{str(dtype)[6:]}_{b}x{n}_{sname}"
                x = torch.randn(b, n, generator=g, dtype=torch.float64).to(dtype)
                if n >= 100:  # ties in the input too
                    x[:, : n // 10] = x[:, n // 10 : 2 * (n // 10)]
                c = torch.randn(b, n, generator=g, dtype=torch.float64).to(dtype)
                xr = x.clone().requires_grad_()
                out = ranks(xr, strength)
                (gx,) = torch.autograd.grad((out * c).sum(), xr)
                arrays[f"{name}/x"] = x.numpy()
                arrays[f"{name}/c"] = c.numpy()
                arrays[f"{name}/out"] = out.detach().numpy()
                arrays[f"{name}/grad"] = gx.numpy()
                meta[name] = {"strength": strength}
    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({len(meta)} cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/torchisotonic-checkout")
    main(sys.argv[1])
