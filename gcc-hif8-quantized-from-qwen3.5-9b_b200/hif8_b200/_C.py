"""Module-level operator functions, the counterpart of the reference's pybind
module ``vllm_ascend_hif8._C`` (reference csrc/extension/pybind.cpp:92-142):
same names, same argument names and defaults (``bias=None``,
``output_dtype=torch.float16``).  Each forwards to the registered
``torch.ops.vllm_ascend_hif8`` operator, whose CUDA implementation is the
C ABI in libhif8_b200.so.
"""

from __future__ import annotations

import torch

from ._loader import load_ops

load_ops()
_ops = torch.ops.vllm_ascend_hif8


def hif8_dynamic_quant(x):
    return _ops.hif8_dynamic_quant(x)


def hif8_static_quant(x, fixed_scale):
    return _ops.hif8_static_quant(x, fixed_scale)


def hif8_scaled_decode(data, scale):
    return _ops.hif8_scaled_decode(data, scale)


def soft_hif8_gemv(activation, weight, token_scale, channel_scale, bias=None, output_dtype=torch.float16):
    return _ops.soft_hif8_gemv(activation, weight, token_scale, channel_scale, bias, output_dtype)


def soft_hif8_gemm(activation, weight, token_scale, channel_scale, bias=None, output_dtype=torch.float16):
    return _ops.soft_hif8_gemm(activation, weight, token_scale, channel_scale, bias, output_dtype)


def soft_hif8_fused_gemm(activation, weight, channel_scale, bias=None, output_dtype=torch.float16):
    return _ops.soft_hif8_fused_gemm(activation, weight, channel_scale, bias, output_dtype)


def soft_hif8_static_fused_gemm(activation, weight, fixed_scale, channel_scale, bias=None,
                                output_dtype=torch.float16):
    return _ops.soft_hif8_static_fused_gemm(activation, weight, fixed_scale, channel_scale, bias, output_dtype)
