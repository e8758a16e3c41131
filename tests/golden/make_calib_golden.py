"""Writes tests/golden/calib.npz: seeded (score, label) sets with the calibration curve and the
calibrated values that the reference's own recipe gives (torchisotonic 0.2.1, imported from a
checkout of it, on the CPU): the pre-step torch.sort -> unique_consecutive -> index_add_ ->
sums / counts, then torchisotonic.isotonic(means, counts), and the reading of new scores by
torch.searchsorted, clamps and a linear interpolation (README.md:43-56 of the reference).

    python tests/golden/make_calib_golden.py /path/to/torchisotonic

Each case stores scores, labels, the curve (xs, fit), new scores x and their values.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "calib.npz"


def main(ref_src: str) -> None:
    sys.path.insert(0, str(Path(ref_src) / "src"))
    import torchisotonic

    def curve(scores: torch.Tensor, labels: torch.Tensor):
        s, order = torch.sort(scores, stable=True)
        xs, inverse, counts = torch.unique_consecutive(s, return_inverse=True,
                                                       return_counts=True)
        sums = torch.zeros(len(xs), dtype=torch.float64)
        sums.index_add_(0, inverse, labels[order].double())
        return xs, torchisotonic.isotonic(sums / counts, counts.double())

    def read(x: torch.Tensor, xs: torch.Tensor, fit: torch.Tensor) -> torch.Tensor:
        i = torch.searchsorted(xs, x).clamp(1, len(xs) - 1)
        t = ((x - xs[i - 1]) / (xs[i] - xs[i - 1])).clamp(0, 1)
        return fit[i - 1] + t * (fit[i] - fit[i - 1])

    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    def add(name: str, scores: torch.Tensor, labels: torch.Tensor, x: torch.Tensor) -> None:
        xs, fit = curve(scores, labels)
        arrays[f"{name}/scores"] = scores.numpy()
        arrays[f"{name}/labels"] = labels.numpy()
        arrays[f"{name}/xs"] = xs.numpy()
        arrays[f"{name}/fit"] = fit.numpy()
        arrays[f"{name}/x"] = x.numpy()
        arrays[f"{name}/read"] = read(x, xs, fit).numpy()
        meta[name] = {"n": scores.numel(), "groups": xs.numel()}

    def probes(scores: torch.Tensor, g: torch.Generator, m: int = 2000) -> torch.Tensor:
        lo, hi = float(scores.min()), float(scores.max())
        span = hi - lo if hi > lo else 1.0
        x = lo - 0.1 * span + 1.2 * span * torch.rand(m, generator=g, dtype=torch.float64)
        extra = torch.tensor([lo, hi, lo - 1.0, hi + 1.0, math.nan, math.inf, -math.inf],
                             dtype=torch.float64)
        pick = scores[torch.randint(scores.numel(), (50,), generator=g)].double()
        return torch.cat([x, extra, pick]).to(scores.dtype)

    g = torch.Generator().manual_seed(11)
    s = torch.tensor([0.3, 0.1, 0.3, 0.2, 0.1])
    add("small", s, torch.tensor([1.0, 0.0, 0.0, 1.0, 1.0]), probes(s, g))
    s = torch.tensor([0.5, 0.5, 0.5])
    add("one_group", s, torch.tensor([1.0, 0.0, 1.0]), probes(s, g))
    s = torch.tensor([2.0])
    add("single", s, torch.tensor([1.0]), probes(s, g))
    s = torch.tensor([0.0, -0.0, 1.0, -0.0, 2.0, 0.0])
    add("signed_zero", s, torch.tensor([1.0, 0.0, 0.0, 1.0, 1.0, 0.0]), probes(s, g))

    # unique model scores with Bernoulli labels (the Criteo example's shape, small)
    s = torch.sigmoid(torch.randn(20000, generator=g))
    lab = torch.bernoulli(s, generator=g)
    add("unique_f32", s, lab, probes(s, g))
    # heavy ties: groups spanning many tiles of the kernels (a tile is 4096 pairs)
    s = torch.randint(0, 300, (50000,), generator=g).float() / 300
    lab = torch.bernoulli(torch.sigmoid(6 * s - 3), generator=g)
    add("ties_300", s, lab, probes(s, g))
    s = torch.randint(0, 5, (40000,), generator=g).float()
    lab = torch.bernoulli(torch.full((40000,), 0.4), generator=g)
    add("ties_5", s, lab, probes(s, g))
    # float64 scores, labels that are not 0/1
    s = torch.randn(30000, generator=g, dtype=torch.float64).round(decimals=2)
    lab = torch.rand(30000, generator=g, dtype=torch.float64)
    add("f64_rates", s, lab, probes(s, g))
    # decreasing trend: the fit pools into few blocks
    s = torch.rand(15000, generator=g)
    lab = torch.bernoulli(1 - s, generator=g)
    add("decreasing", s, lab, probes(s, g))

    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({len(meta)} cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/torchisotonic-checkout")
    main(sys.argv[1])
