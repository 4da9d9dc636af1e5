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


def channel_rel(actual: np.ndarray, expected: np.ndarray, floor_frac: float = 1e-3) -> float:
    """Worst per-output-channel relative error: for every channel (last axis)
    max over rows |actual - expected| divided by that channel's own max
    |expected|, so a wrong small-magnitude channel cannot hide under the
    largest output of the tensor.  A channel whose outputs are all below
    floor_frac x the tensor's max |expected| is measured against that floor
    (a relative error of values near zero says nothing about the kernel)."""
    actual = np.asarray(actual, np.float64).reshape(-1, np.shape(actual)[-1])
    expected = np.asarray(expected, np.float64).reshape(-1, np.shape(expected)[-1])
    floor = max(float(np.abs(expected).max()) * floor_frac, 1e-30)
    denom = np.maximum(np.abs(expected).max(axis=0), floor)
    return float((np.abs(actual - expected).max(axis=0) / denom).max())


def row_cosine_min(actual: np.ndarray, expected: np.ndarray) -> float:
    """Smallest cosine similarity between matching rows (first axes
    flattened) of actual and expected."""
    a = np.asarray(actual, np.float64).reshape(-1, np.shape(actual)[-1])
    e = np.asarray(expected, np.float64).reshape(-1, np.shape(expected)[-1])
    num = (a * e).sum(axis=1)
    den = np.maximum(np.linalg.norm(a, axis=1) * np.linalg.norm(e, axis=1), 1e-300)
    return float((num / den).min())
