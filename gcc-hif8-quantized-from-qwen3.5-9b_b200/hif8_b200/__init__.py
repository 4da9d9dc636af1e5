"""hif8_b200: B200 (sm_100a) HiFloat8 static W8A8KV8 hot path.

Drop-in for the HiF8 operators of the reference vLLM-Ascend plugin:
``torch.ops.vllm_ascend_hif8.{hif8_static_quant, hif8_scaled_decode,
soft_hif8_gemv, soft_hif8_gemm, soft_hif8_static_fused_gemm}`` plus the fused
paged-KV operators ``torch.ops.hif8_b200.*``.  Kernels live in
``libhif8_b200.so`` (C ABI, include/hif8_b200.h); ``native`` mirrors the
reference's Python operator boundary.
"""

from ._loader import NativeExtensionUnavailable, load_ops

__all__ = ["NativeExtensionUnavailable", "load_ops"]
__version__ = "0.1.0"
