"""Shared test set-up: the `gpu` marker, the repository root on sys.path, golden fixtures."""

from __future__ import annotations

import json
import sys
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.npz"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@lru_cache(maxsize=1)
def golden() -> tuple[dict, dict]:
    """(meta, arrays) of the reference-generated fixtures (tests/golden/make_golden.py)."""
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["__meta__"]).decode())
    arrays = {k: z[k] for k in z.files if k != "__meta__"}
    return meta, arrays


def golden_case(name: str) -> dict:
    meta, arrays = golden()
    case = dict(meta[name])
    prefix = name + "/"
    for k, v in arrays.items():
        if k.startswith(prefix):
            case[k[len(prefix):]] = v
    return case


def golden_names(pred=lambda name, meta: True) -> list[str]:
    meta, _ = golden()
    return [k for k, m in meta.items() if pred(k, m)]
