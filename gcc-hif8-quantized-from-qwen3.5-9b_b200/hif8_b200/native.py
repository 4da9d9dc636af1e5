"""Python operator boundary, the B200 counterpart of the reference's
``vllm_ascend_hif8.native`` (reference src/vllm_ascend_hif8/native.py).

Same functions, argument checks, exception types and GEMV/GEMM routing; the
operators underneath are the sm_100a kernels behind
``torch.ops.vllm_ascend_hif8.*``.  There is no CPU or decoded-weight
fallback: a missing extension raises ``NativeExtensionUnavailable``.
"""

from __future__ import annotations

import os
from types import ModuleType
from typing import TYPE_CHECKING

from ._loader import NativeExtensionUnavailable, load_ops, reset as _reset_loader

if TYPE_CHECKING:
    import torch

_REQUIRED_SYMBOLS = (
    "hif8_dynamic_quant",
    "hif8_static_quant",
    "hif8_scaled_decode",
    "soft_hif8_gemv",
    "soft_hif8_gemm",
    "soft_hif8_static_fused_gemm",
)
_extension: ModuleType | None = None
_load_error: BaseException | None = None

# Reference routing limits (native.py:22-25): the GEMV operator keeps its
# narrow-N, short-K, single-row contract; everything else is soft_hif8_gemm,
# which itself runs the split-K tensor-core GEMV for M <= 16.
_SOFT_HIF8_GEMV_MAX_OUTPUT_COLUMNS = 1_536
_SOFT_HIF8_GEMV_MAX_INPUT_COLUMNS = 8_192
_DISABLE_GEMV_ENV = "HIF8_DISABLE_GEMV"

__all__ = [
    "NativeExtensionUnavailable",
    "dynamic_quant",
    "is_available",
    "load_extension",
    "reset_extension_cache",
    "scaled_decode",
    "soft_fused_linear",
    "soft_linear",
    "soft_static_fused_linear",
    "static_quant",
]


def load_extension() -> ModuleType:
    """Load and validate the native extension, caching success or failure
    (reference native.py:32-50)."""
    global _extension, _load_error
    if _extension is not None:
        return _extension
    if _load_error is not None:
        raise NativeExtensionUnavailable(_error_message()) from _load_error
    try:
        load_ops()
        from . import _C as candidate

        missing = [s for s in _REQUIRED_SYMBOLS if not callable(getattr(candidate, s, None))]
        if missing:
            raise ImportError(f"native extension is missing required symbols: {', '.join(missing)}")
        _extension = candidate
        return candidate
    except BaseException as error:
        _load_error = error
        raise NativeExtensionUnavailable(_error_message()) from error


def _error_message() -> str:
    if isinstance(_load_error, NativeExtensionUnavailable):
        return str(_load_error)
    detail = f": {_load_error}" if _load_error is not None else ""
    return (
        "B200 HiFloat8 native operators are unavailable"
        f"{detail}. Build them with gcc-hif8-quantized-from-qwen3.5-9b_b200/build.py; "
        "the production path intentionally has no decoded-weight or floating-point fallback."
    )


def is_available() -> bool:
    try:
        load_extension()
    except NativeExtensionUnavailable:
        return False
    return True


def reset_extension_cache() -> None:
    """Reset loader state for isolated tests."""
    global _extension, _load_error, _static_linear_op
    _extension = None
    _load_error = None
    _static_linear_op = None
    _OPS.clear()
    _reset_loader()


_OPS: dict = {}


def _op(name: str):
    """The registered operator (resolved once per name)."""
    operator = _OPS.get(name)
    if operator is not None:
        return operator
    import torch

    extension = load_extension()
    operator = getattr(torch.ops.vllm_ascend_hif8, name, None)
    if operator is None:
        operator = getattr(extension, name, None)
    if not callable(operator):
        raise NativeExtensionUnavailable(f"the native extension has no {name} operator")
    _OPS[name] = operator
    return operator


def dynamic_quant(x: "torch.Tensor") -> tuple["torch.Tensor", "torch.Tensor"]:
    """Quantize BF16/FP16 activations into U8 HiFloat8 with one FP32 scale
    per row (the row's finite amax, at least 1e-12) -- the W8A8HIF8_SOFT
    activation path (reference native.py:77-87); the scales come back as the
    reference's stride-16 view."""
    load_extension()
    data, scale = _op("hif8_dynamic_quant")(x)
    _validate_quantized_activation(x, data, scale, operation="hif8_dynamic_quant")
    return data, scale


def static_quant(x: "torch.Tensor", fixed_scale: "torch.Tensor") -> tuple["torch.Tensor", "torch.Tensor"]:
    """Quantize with fixed FP32 scale(s), without an activation reduction
    (reference native.py:90-124).

    One scale is used for every row in a Linear activation.  For KV tensors,
    flatten ``[tokens, heads, dim]`` into ``[tokens * heads, dim]`` and pass one
    scale per head; row r uses scale[r % heads].
    """
    import torch

    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"static HiFloat8 quant requires FP16/BF16 input, got {x.dtype}")
    if x.ndim < 1:
        raise ValueError("static HiFloat8 quant requires at least one dimension")
    if fixed_scale.dtype != torch.float32 or fixed_scale.ndim != 1:
        raise TypeError("fixed_scale must be a 1D torch.float32 tensor")
    rows = x.numel() // x.shape[-1]
    if fixed_scale.numel() <= 0 or rows % fixed_scale.numel():
        raise ValueError(f"fixed_scale count {fixed_scale.numel()} must divide {rows} activation rows")
    if fixed_scale.device != x.device:
        raise ValueError(f"fixed_scale must be on {x.device}, got {fixed_scale.device}")
    x = _as_native_operand(x)
    fixed_scale = _as_native_operand(fixed_scale)
    data, scale = _op("hif8_static_quant")(x, fixed_scale)
    _validate_quantized_activation(x, data, scale, operation="hif8_static_quant")
    return data, scale


def scaled_decode(data: "torch.Tensor", scale: "torch.Tensor") -> "torch.Tensor":
    """Decode U8 HiFloat8 rows with FP32 scales into a BF16 tensor
    (reference native.py:127-145)."""
    import torch

    if data.dtype != torch.uint8:
        raise TypeError(f"scaled_decode requires uint8 data, got {data.dtype}")
    if scale.dtype != torch.float32:
        raise TypeError(f"scaled_decode requires float32 scale, got {scale.dtype}")
    if data.ndim != 2:
        raise ValueError(f"scaled_decode requires 2D data, got shape {data.shape}")
    load_extension()
    data = _as_native_operand(data)
    scale = _as_native_operand(scale.reshape(-1))
    return _op("hif8_scaled_decode")(data, scale)


def _flat2d(tensor: "torch.Tensor") -> "torch.Tensor":
    """[..., K] -> [rows, K] (no new view when already 2-D)."""
    return tensor if tensor.dim() == 2 else tensor.reshape(-1, tensor.shape[-1])


def _flat1d(tensor: "torch.Tensor") -> "torch.Tensor":
    return tensor if tensor.dim() == 1 else tensor.reshape(-1)


def _as_native_operand(tensor: "torch.Tensor") -> "torch.Tensor":
    """Return a tensor the native bridge accepts (contiguous, zero offset)
    (reference native.py:148-157)."""
    if tensor.is_contiguous() and tensor.storage_offset() == 0:
        return tensor
    return tensor.contiguous().clone()


def soft_linear(
    activation: "torch.Tensor",
    weight: "torch.Tensor",
    activation_scale: "torch.Tensor",
    weight_scale: "torch.Tensor",
    bias: "torch.Tensor | None" = None,
    *,
    output_dtype: "torch.dtype",
) -> "torch.Tensor":
    """Dispatch physical U8 operands to the GEMV or GEMM operator
    (reference native.py:160-201)."""
    import torch

    if activation.dtype != torch.uint8 or weight.dtype != torch.uint8:
        raise TypeError("soft HiFloat8 linear requires uint8 activation and weight tensors")
    if activation.ndim < 2 or weight.ndim != 2:
        raise ValueError("activation must be at least 2D and weight must be 2D")
    if activation.shape[-1] != weight.shape[-1]:
        raise ValueError(f"incompatible K dimensions: activation={activation.shape[-1]}, weight={weight.shape[-1]}")
    if activation_scale.dtype != torch.float32 or weight_scale.dtype != torch.float32:
        raise TypeError("soft HiFloat8 linear requires float32 activation and weight scales")

    load_extension()
    flattened = _as_native_operand(_flat2d(activation))
    token_scale = _as_native_operand(_flat1d(activation_scale))
    channel_scale = _as_native_operand(_flat1d(weight_scale))
    if token_scale.numel() != flattened.shape[0]:
        raise ValueError("activation_scale must contain one value per token row")
    if channel_scale.numel() != weight.shape[0]:
        raise ValueError("weight_scale must contain one value per output channel")

    use_gemv = (
        os.environ.get(_DISABLE_GEMV_ENV) != "1"
        and flattened.shape[0] == 1
        and weight.shape[0] <= _SOFT_HIF8_GEMV_MAX_OUTPUT_COLUMNS
        and flattened.shape[1] <= _SOFT_HIF8_GEMV_MAX_INPUT_COLUMNS
    )
    operator = _op("soft_hif8_gemv" if use_gemv else "soft_hif8_gemm")
    output = operator(flattened, weight, token_scale, channel_scale, bias, output_dtype)
    return output if activation.dim() == 2 else output.reshape(*activation.shape[:-1], weight.shape[0])


def soft_fused_linear(
    x: "torch.Tensor",
    weight: "torch.Tensor",
    weight_scale: "torch.Tensor",
    bias: "torch.Tensor | None" = None,
    *,
    output_dtype: "torch.dtype",
) -> "torch.Tensor":
    """Dynamic activation quant fused with the U8-weight linear, M <= 2
    (reference native.py:204-240; the result equals dynamic_quant then
    soft_linear bit for bit)."""
    import torch

    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"fused soft HiFP8 linear requires FP16/BF16 activation, got {x.dtype}")
    if weight.dtype != torch.uint8 or weight.ndim != 2:
        raise TypeError("fused soft HiFP8 linear requires a 2D uint8 weight tensor")
    if x.ndim < 2 or x.shape[-1] != weight.shape[-1]:
        raise ValueError("activation and weight must have compatible final K dimensions")
    if weight_scale.dtype != torch.float32 or weight_scale.numel() != weight.shape[0]:
        raise TypeError("fused soft HiFP8 linear requires one float32 scale per output channel")
    flattened = _as_native_operand(x.reshape(-1, x.shape[-1]))
    if flattened.shape[0] > 2:
        raise ValueError("fused soft HiFP8 linear supports M <= 2")
    channel_scale = _as_native_operand(weight_scale.reshape(-1))
    load_extension()
    output = _op("soft_hif8_fused_gemm")(flattened, weight, channel_scale, bias, output_dtype)
    return output.reshape(*x.shape[:-1], weight.shape[0])


def soft_static_fused_linear(
    x: "torch.Tensor",
    weight: "torch.Tensor",
    fixed_scale: "torch.Tensor",
    weight_scale: "torch.Tensor",
    bias: "torch.Tensor | None" = None,
    *,
    output_dtype: "torch.dtype",
) -> "torch.Tensor":
    """Fixed-scale activation encode/decode fused with the U8-weight linear
    (reference native.py:241-284)."""
    import torch

    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"static fused soft HiFP8 linear requires FP16/BF16 activation, got {x.dtype}")
    if weight.dtype != torch.uint8 or weight.ndim != 2:
        raise TypeError("static fused soft HiFP8 linear requires a 2D uint8 weight tensor")
    if x.ndim < 2 or x.shape[-1] != weight.shape[-1]:
        raise ValueError("activation and weight must have compatible final K dimensions")
    if fixed_scale.dtype != torch.float32 or fixed_scale.ndim != 1 or fixed_scale.numel() != 1:
        raise TypeError("static fused soft HiFP8 linear requires one float32 activation scale")
    if weight_scale.dtype != torch.float32 or weight_scale.numel() != weight.shape[0]:
        raise TypeError("static fused soft HiFP8 linear requires one float32 scale per output channel")
    device = x.device
    if fixed_scale.device != device or weight_scale.device != device or weight.device != device:
        raise ValueError("activation, weight, fixed_scale, and weight_scale must be on the same device")

    load_extension()
    flattened = _as_native_operand(_flat2d(x))
    fixed = _as_native_operand(fixed_scale)
    channel_scale = _as_native_operand(_flat1d(weight_scale))
    output = _op("soft_hif8_static_fused_gemm")(flattened, weight, fixed, channel_scale, bias, output_dtype)
    return output if x.dim() == 2 else output.reshape(*x.shape[:-1], weight.shape[0])


_static_linear_op = None


def static_linear(x, weight, input_scale, weight_scale, bias=None, fused_max_rows: int = 4):
    """Static quant + HiF8 linear as ONE operator (hif8_b200::static_linear),
    output in x's dtype: the pair of calls the static scheme's apply makes,
    routed in the operator.  The operator checks its arguments with the
    messages of the two reference operators it replaces."""
    global _static_linear_op
    op = _static_linear_op
    if op is None:
        import torch

        load_extension()
        op = _static_linear_op = torch.ops.hif8_b200.static_linear.default
    return op(x, weight, input_scale, weight_scale, bias, fused_max_rows)


def _validate_quantized_activation(source, data, scale, *, operation: str = "hif8_static_quant") -> None:
    import torch

    if data.dtype != torch.uint8:
        raise RuntimeError(f"{operation} returned {data.dtype}, expected torch.uint8")
    if data.shape != source.shape:
        raise RuntimeError(f"{operation} changed activation shape from {source.shape} to {data.shape}")
    if scale.dtype != torch.float32:
        raise RuntimeError(f"{operation} returned {scale.dtype} scale, expected torch.float32")
    expected_rows = source.numel() // source.shape[-1]
    if scale.numel() != expected_rows:
        raise RuntimeError(f"{operation} returned {scale.numel()} scales for {expected_rows} activation rows")
