"""Shared pytest configuration.

The product package lives in ``gcc-hif8-quantized-from-qwen3.5-9b_b200/`` (a
folder name that is not a Python identifier), so that folder is put on
``sys.path`` and the package is imported as ``hif8_b200``.  The repository
root is put on ``sys.path`` for the ``oracle`` checker.
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "gcc-hif8-quantized-from-qwen3.5-9b_b200"
for path in (str(ROOT), str(PKG_ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import pytest

    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch is part of the image
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
