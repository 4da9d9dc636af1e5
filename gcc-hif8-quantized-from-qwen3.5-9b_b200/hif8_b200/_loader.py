"""Locate and load the native libraries built in place by ``build.py``.

There is no fallback: if a library is missing, every entry point raises
``NativeExtensionUnavailable`` (the production policy of the reference,
src/vllm_ascend_hif8/native.py:28-59).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CABI_PATH = PKG_DIR / "libhif8_b200.so"
OPS_PATH = PKG_DIR / "_C_ops.so"

_lock = threading.Lock()
_ops_loaded = False
_ops_error: BaseException | None = None


class NativeExtensionUnavailable(RuntimeError):
    """Raised when production HiFloat8 execution cannot load native operators."""


def _message(detail: BaseException | None) -> str:
    suffix = f": {detail}" if detail is not None else ""
    return (
        "B200 HiFloat8 native operators are unavailable"
        f"{suffix}. Build them with `python gcc-hif8-quantized-from-qwen3.5-9b_b200/build.py`; "
        "the production path intentionally has no decoded-weight or floating-point fallback."
    )


def load_ops() -> None:
    """Register torch.ops.vllm_ascend_hif8.* and torch.ops.hif8_b200.* (once)."""
    global _ops_loaded, _ops_error
    if _ops_loaded:
        return
    with _lock:
        if _ops_loaded:
            return
        if _ops_error is not None:
            raise NativeExtensionUnavailable(_message(_ops_error)) from _ops_error
        try:
            import torch

            if not OPS_PATH.exists():
                raise FileNotFoundError(f"{OPS_PATH} is not built")
            torch.ops.load_library(str(OPS_PATH))
            _ops_loaded = True
        except BaseException as error:  # cached like the reference loader
            _ops_error = error
            raise NativeExtensionUnavailable(_message(error)) from error


def reset() -> None:
    """Forget a cached load failure (tests only; a loaded library stays loaded)."""
    global _ops_error
    _ops_error = None


def cabi_library() -> ctypes.CDLL:
    """The C-ABI library (include/hif8_b200.h) with argument types declared."""
    from . import cabi

    return cabi.library()
