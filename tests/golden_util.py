"""Turns golden fixtures back into torch tensors (bfloat16 is stored as uint16 bits)."""

from __future__ import annotations

import numpy as np
import torch

DTYPES = {
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "float64": torch.float64,
    "int64": torch.int64,
}


def tensor(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bfloat16" and a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(np.array(a))


def out_tensor(case: dict) -> torch.Tensor:
    dt = case["dtype"]
    a = case["out"]
    if dt == "bfloat16":
        return tensor(a, dt)
    return torch.from_numpy(np.array(a))
