"""Helpers shared by the tests (not collected)."""

from __future__ import annotations

import numpy as np


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(bits: np.ndarray, dtype):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(dtype)


def max_rel(actual: np.ndarray, expected: np.ndarray) -> float:
    denom = max(float(np.abs(expected).max()), 1e-12)
    return float(np.abs(actual - expected).max()) / denom
