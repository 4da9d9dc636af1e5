"""W8A8HIF8_STATIC and W8A8HIF8_SOFT linears: the parameter contracts and
``apply`` of the reference quant schemes (src/vllm_ascend_hif8/scheme.py:134-211
static, 43-132 dynamic) without the vLLM-Ascend registration layer.

Parameters of a layer:
  ``weight``       uint8 [N, K] HiF8 bytes (row-major, K contiguous)
  ``weight_scale`` float32 [N, 1] (flattened to [N] after loading)
  ``input_scale``  float32 [1], positive and finite, fixed for every call
                   (static scheme only; the dynamic scheme computes one
                   scale per token row from its amax)
"""

from __future__ import annotations

import math
import os

from . import native

STATIC_QUANT_TYPE = "W8A8HIF8_STATIC"
DYNAMIC_QUANT_TYPE = "W8A8HIF8_SOFT"
_STATIC_FUSED_GENERATION_ENV = "HIF8_STATIC_FUSED_GENERATION"
_SOFT_FUSED_GENERATION_ENV = "HIF8_SOFT_FUSED_GENERATION"
_STATIC_SCALE_FACTOR_ENV = "HIF8_STATIC_SCALE_FACTOR"
_COMPUTE_BACKEND_ENV = "HIF8_COMPUTE_BACKEND"
MAX_FINITE = 32768.0

# The fused quant+linear kernel serves decode rows (reference policy,
# scheme.py:185-189); on B200 it is cheaper than quant + linear at every K,
# so it is the default for rows <= 4 unless HIF8_STATIC_FUSED_GENERATION=0.
_FUSED_MAX_ROWS = 4
# The dynamic fused kernel is opt-in (HIF8_SOFT_FUSED_GENERATION=1) for at
# most two token rows, as in the reference (scheme.py:101-109).
_SOFT_FUSED_MAX_ROWS = 2


# (raw environment string, parsed factor) of the last valid read: apply
# re-reads the variable on every call, and parses it only when it changed
_factor_cache: tuple = (None, 1.0)


def static_scale_factor() -> float:
    """Optional constant multiplier of calibrated input scales (scheme.py:26-40)."""
    global _factor_cache
    raw = os.environ.get(_STATIC_SCALE_FACTOR_ENV)
    if raw == _factor_cache[0]:
        return _factor_cache[1]
    if raw is None or raw == "":
        return 1.0
    try:
        value = float(raw)
    except ValueError as exc:
        raise ValueError(f"{_STATIC_SCALE_FACTOR_ENV} must be a positive finite float") from exc
    if not math.isfinite(value) or value <= 0.0:
        raise ValueError(f"{_STATIC_SCALE_FACTOR_ENV} must be a positive finite float")
    _factor_cache = (raw, value)
    return value


def _check_backend() -> None:
    backend = os.environ.get(_COMPUTE_BACKEND_ENV, "soft_hif8")
    if backend != "soft_hif8":
        raise ValueError(f"{_COMPUTE_BACKEND_ENV} must be 'soft_hif8', got {backend!r}")


def process_weights_after_loading(layer) -> None:
    """Validate and normalise a loaded layer in place (scheme.py:157-172 and
    the weight handling of scheme.py:59-91)."""
    import torch

    _check_backend()
    if not hasattr(layer, "input_scale"):
        raise ValueError(f"{STATIC_QUANT_TYPE} checkpoint is missing input_scale")
    scale = layer.input_scale.data.to(dtype=torch.float32).reshape(-1)
    if scale.numel() != 1:
        raise ValueError(f"{STATIC_QUANT_TYPE} requires one input_scale value, got "
                         f"shape {tuple(layer.input_scale.shape)}")
    if not bool(torch.isfinite(scale).all()) or not bool((scale > 0).all()):
        raise ValueError(f"{STATIC_QUANT_TYPE} input_scale must be finite and greater than zero")
    layer.input_scale.data = scale.contiguous()
    if layer.weight.dtype != torch.uint8 or layer.weight.ndim != 2:
        raise ValueError(f"{STATIC_QUANT_TYPE} weight must be a 2D uint8 tensor")
    layer.weight.data = layer.weight.data.contiguous()
    ws = layer.weight_scale.data.to(torch.float32).reshape(-1)
    if ws.numel() != layer.weight.shape[0]:
        raise ValueError("weight_scale must contain one value per output channel")
    layer.weight_scale.data = ws.contiguous()


def apply(layer, x, bias=None):
    """Static activation quant + HiF8 linear (scheme.py:174-211) in one
    operator call: the operator takes the fused quant + linear for rows <= 4
    (unless HIF8_STATIC_FUSED_GENERATION=0), else the static quant and then
    the linear -- the kernels of native.soft_static_fused_linear /
    native.static_quant + native.soft_linear, with the same bytes -- so the
    routing costs no extra dispatch.  The layer's parameters were validated
    when it was loaded (process_weights_after_loading)."""
    fused_rows = 0 if os.environ.get(_STATIC_FUSED_GENERATION_ENV) == "0" else _FUSED_MAX_ROWS
    fixed_scale = layer.input_scale
    factor = static_scale_factor()
    if factor != 1.0:
        fixed_scale = fixed_scale * factor
    return native.static_linear(x, layer.weight, fixed_scale, layer.weight_scale, bias, fused_rows)


def process_dynamic_weights_after_loading(layer) -> None:
    """Validate and normalise a loaded W8A8HIF8_SOFT layer in place
    (scheme.py:56-91): uint8 weight, FP32 per-channel scale flattened to
    [N]; no input_scale."""
    import torch

    if layer.weight.dtype != torch.uint8:
        raise TypeError(f"{DYNAMIC_QUANT_TYPE} checkpoint weight must be torch.uint8, got {layer.weight.dtype}")
    if layer.weight.ndim != 2:
        raise ValueError(f"{DYNAMIC_QUANT_TYPE} weight must be a 2D uint8 tensor")
    layer.weight.data = layer.weight.data.contiguous()
    ws = layer.weight_scale.data.to(torch.float32).reshape(-1)
    if ws.numel() != layer.weight.shape[0]:
        raise ValueError("weight_scale must contain one value per output channel")
    layer.weight_scale.data = ws.contiguous()
    _check_backend()


def apply_dynamic(layer, x, bias=None):
    """Dynamic per-token activation quant + HiF8 linear (scheme.py:93-116)."""
    token_rows = x.numel() // x.shape[-1]
    if token_rows <= _SOFT_FUSED_MAX_ROWS and os.environ.get(_SOFT_FUSED_GENERATION_ENV) == "1":
        return native.soft_fused_linear(x, layer.weight, layer.weight_scale, bias, output_dtype=x.dtype)
    activation, row_scale = native.dynamic_quant(x)
    return native.soft_linear(activation, layer.weight, row_scale, layer.weight_scale, bias, output_dtype=x.dtype)


def quantize_weight_rows(weight, scale_factor: float = MAX_FINITE):
    """Per-output-channel HiF8 weight quantisation on the device:
    scale = max(row amax, 1e-12) / scale_factor and bytes = encode(w / scale)
    -- the export rule of torch_codec.quantize_tensor_rows (reference
    torch_codec.py:52-73) run through the static quantiser (row r uses
    scale[r]).  Bytes are identical because |w / scale| <= scale_factor."""
    import torch

    w = weight.contiguous()
    amax = w.float().abs().amax(dim=-1)
    scale = (amax.clamp(min=1.0e-12) / scale_factor).to(torch.float32).contiguous()
    data, _ = native.static_quant(w, scale)
    return data, scale


class Hif8StaticLinear:
    """A standalone W8A8HIF8_STATIC projection holding device parameters."""

    def __init__(self, weight, weight_scale, input_scale, bias=None):
        import torch

        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.weight_scale = torch.nn.Parameter(weight_scale, requires_grad=False)
        self.input_scale = torch.nn.Parameter(input_scale, requires_grad=False)
        self.bias = bias
        process_weights_after_loading(self)

    @classmethod
    def from_float(cls, weight, input_scale, bias=None, scale_factor: float = MAX_FINITE):
        data, scale = quantize_weight_rows(weight, scale_factor)
        return cls(data, scale.reshape(-1, 1), input_scale, bias)

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1]

    def __call__(self, x):
        return apply(self, x, self.bias)


class Hif8SoftLinear:
    """A standalone W8A8HIF8_SOFT projection: per-channel HiF8 weights and a
    per-token activation scale computed on every call."""

    def __init__(self, weight, weight_scale, bias=None):
        import torch

        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.weight_scale = torch.nn.Parameter(weight_scale, requires_grad=False)
        self.bias = bias
        process_dynamic_weights_after_loading(self)

    @classmethod
    def from_float(cls, weight, bias=None, scale_factor: float = MAX_FINITE):
        data, scale = quantize_weight_rows(weight, scale_factor)
        return cls(data, scale.reshape(-1, 1), bias)

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1]

    def __call__(self, x):
        return apply_dynamic(self, x, self.bias)
