"""ctypes binding of the C ABI declared in include/hif8_b200.h.

This is the binding a non-PyTorch host would write; the PyTorch operators in
``_C_ops.so`` call the same entry points from C++.  The helpers below accept
torch tensors only for their device pointers and the current CUDA stream.
"""

from __future__ import annotations

import ctypes
import threading

from ._loader import CABI_PATH, NativeExtensionUnavailable

HIF8_OK = 0
HIF8_ERR_INVALID_ARGUMENT = 1
HIF8_ERR_CUDA = 2
HIF8_ERR_WORKSPACE = 3

HIF8_DTYPE_F16 = 0
HIF8_DTYPE_BF16 = 1
HIF8_DTYPE_NONE = -1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); one entry per declaration in include/hif8_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "hif8_status_string": (ctypes.c_char_p, [_INT]),
    "hif8_last_error": (ctypes.c_char_p, []),
    "hif8_version": (ctypes.c_char_p, []),
    "hif8_decode_table_bf16": (None, [_P]),
    "hif8_encode_table": (None, [_P]),
    "hif8_static_quant": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _P, _P]),
    "hif8_scaled_decode": (_INT, [_P, _I64, _I64, _I64, _P, _P, _P]),
    "hif8_embedding_gather": (_INT, [_P, _P, _I64, _I64, _P, _I64, _P, _P, _P]),
    "soft_hif8_gemv": (_INT, [_P, _P, _P, _P, _P, _INT, _INT, _I64, _I64, _I64, _P, _P]),
    "soft_hif8_gemm_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "soft_hif8_gemm": (_INT, [_P, _P, _P, _P, _P, _INT, _INT, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "hif8_linear_partial_f32": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "hif8_dynamic_quant": (_INT, [_P, _INT, _I64, _I64, _P, _P, _I64, _P]),
    "soft_hif8_fused_gemm_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "soft_hif8_fused_gemm": (_INT, [_P, _INT, _P, _P, _P, _INT, _INT, _I64, _I64, _I64, _P, _P, _SZ, _P]),
    "hif8_static_linear_workspace_size": (_SZ, [_I64, _I64, _I64, _INT]),
    "hif8_static_linear": (_INT, [_P, _INT, _P, _P, _P, _P, _INT, _INT, _I64, _I64, _I64, _INT, _P, _P, _SZ, _P]),
    "hif8_static_fused_linear_partial_f32": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "soft_hif8_static_fused_gemm": (_INT, [_P, _INT, _P, _P, _P, _P, _INT, _INT, _I64, _I64, _I64, _P, _P]),
    "hif8_kv_cache_write": (_INT, [_P, _P, _INT, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _P]),
    "hif8_kv_cache_write_strided": (_INT, [_P, _P, _INT, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                           _P, _P]),
    "hif8_paged_attention_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "hif8_paged_attention": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                    ctypes.c_float, _INT, _P, _P, _SZ, _P]),
    "hif8_paged_attention_strided": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                            _I64, _I64, ctypes.c_float, _INT, _P, _P, _SZ, _P]),
    "hif8_paged_attention_noalloc": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                            _I64, ctypes.c_float, _INT, _P, _P]),
    "hif8_kv_gather_decode": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P]),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def library() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not CABI_PATH.exists():
                raise NativeExtensionUnavailable(f"{CABI_PATH} is not built")
            lib = ctypes.CDLL(str(CABI_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


class Hif8Error(RuntimeError):
    def __init__(self, name: str, status: int):
        lib = library()
        text = lib.hif8_status_string(status).decode()
        if status == HIF8_ERR_CUDA:
            text += f" ({lib.hif8_last_error().decode()})"
        super().__init__(f"{name} failed: {text}")
        self.status = status


def check(name: str, status: int) -> None:
    if status != HIF8_OK:
        raise Hif8Error(name, status)


# ------------------------------------------------------------ helpers ---

def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t) -> int:
    import torch

    return torch.cuda.current_stream(t.device).cuda_stream


def _dtype_code(dtype) -> int:
    import torch

    if dtype == torch.bfloat16:
        return HIF8_DTYPE_BF16
    if dtype == torch.float16:
        return HIF8_DTYPE_F16
    raise TypeError(f"expected torch.float16 or torch.bfloat16, got {dtype}")


def static_quant(x, fixed_scale, data, row_scale=None) -> None:
    k = x.shape[-1]
    rows = x.numel() // k
    check("hif8_static_quant", library().hif8_static_quant(
        _ptr(x), _dtype_code(x.dtype), rows, k, _ptr(fixed_scale), fixed_scale.numel(), _ptr(data),
        _ptr(row_scale), _stream(x)))


def scaled_decode(data, scale, out, row_stride: int | None = None) -> None:
    rows, k = out.shape
    check("hif8_scaled_decode", library().hif8_scaled_decode(
        _ptr(data), rows, k, k if row_stride is None else row_stride, _ptr(scale), _ptr(out), _stream(out)))


def embedding_gather(weight, weight_scale, ids, out, bad_ids=None) -> None:
    vocab, k = weight.shape
    check("hif8_embedding_gather", library().hif8_embedding_gather(
        _ptr(weight), _ptr(weight_scale), vocab, k, _ptr(ids), ids.numel(), _ptr(out), _ptr(bad_ids), _stream(out)))


def gemm(activation, weight, token_scale, channel_scale, bias, out, workspace=None) -> None:
    m, k = activation.shape
    n = weight.shape[0]
    lib = library()
    need = lib.soft_hif8_gemm_workspace_size(m, n, k)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if need and workspace is None:
        import torch

        workspace = torch.empty(need, dtype=torch.uint8, device=activation.device)
        ws_bytes = need
    check("soft_hif8_gemm", lib.soft_hif8_gemm(
        _ptr(activation), _ptr(weight), _ptr(token_scale), _ptr(channel_scale), _ptr(bias),
        HIF8_DTYPE_NONE if bias is None else _dtype_code(bias.dtype), _dtype_code(out.dtype), m, n, k, _ptr(out),
        _ptr(workspace), ws_bytes, _stream(out)))


def static_linear(x, weight, input_scale, channel_scale, bias, out, fused_max_rows: int = 4, workspace=None) -> None:
    """The static scheme's quant + linear pair in one C-ABI call."""
    k = x.shape[-1]
    m = x.numel() // k
    n = weight.shape[0]
    lib = library()
    need = lib.hif8_static_linear_workspace_size(m, n, k, fused_max_rows)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if need and workspace is None:
        import torch

        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
        ws_bytes = need
    check("hif8_static_linear", lib.hif8_static_linear(
        _ptr(x), _dtype_code(x.dtype), _ptr(weight), _ptr(input_scale), _ptr(channel_scale), _ptr(bias),
        HIF8_DTYPE_NONE if bias is None else _dtype_code(bias.dtype), _dtype_code(out.dtype), m, n, k,
        fused_max_rows, _ptr(out), _ptr(workspace), ws_bytes, _stream(out)))


def gemv(activation, weight, token_scale, channel_scale, bias, out) -> None:
    m, k = activation.shape
    n = weight.shape[0]
    check("soft_hif8_gemv", library().soft_hif8_gemv(
        _ptr(activation), _ptr(weight), _ptr(token_scale), _ptr(channel_scale), _ptr(bias),
        HIF8_DTYPE_NONE if bias is None else _dtype_code(bias.dtype), _dtype_code(out.dtype), m, n, k, _ptr(out),
        _stream(out)))


def static_fused_gemm(x, weight, fixed_scale, channel_scale, bias, out) -> None:
    m, k = x.shape
    n = weight.shape[0]
    check("soft_hif8_static_fused_gemm", library().soft_hif8_static_fused_gemm(
        _ptr(x), _dtype_code(x.dtype), _ptr(weight), _ptr(fixed_scale), _ptr(channel_scale), _ptr(bias),
        HIF8_DTYPE_NONE if bias is None else _dtype_code(bias.dtype), _dtype_code(out.dtype), m, n, k, _ptr(out),
        _stream(out)))


def kv_cache_write(key, value, key_scale, value_scale, slot_mapping, key_cache, value_cache, bad_slots=None) -> None:
    tokens, heads, d = key.shape
    if key_cache.stride(0) != key_cache[0].numel() and key_cache.shape[0] > 1:
        check("hif8_kv_cache_write_strided", library().hif8_kv_cache_write_strided(
            _ptr(key), _ptr(value), _dtype_code(key.dtype), tokens, heads, d, key.stride(0), _ptr(key_scale),
            _ptr(value_scale), _ptr(slot_mapping), _ptr(key_cache), _ptr(value_cache), key_cache.shape[0],
            key_cache.shape[1], key_cache.stride(0), _ptr(bad_slots), _stream(key)))
        return
    check("hif8_kv_cache_write", library().hif8_kv_cache_write(
        _ptr(key), _ptr(value), _dtype_code(key.dtype), tokens, heads, d, key.stride(0), _ptr(key_scale),
        _ptr(value_scale), _ptr(slot_mapping), _ptr(key_cache), _ptr(value_cache), key_cache.shape[0],
        key_cache.shape[1], _ptr(bad_slots), _stream(key)))


def paged_attention(query, key_cache, value_cache, block_tables, seq_lens, query_start, max_seq_len, scale,
                    out, causal: bool = True, workspace=None) -> None:
    import torch

    tokens, heads, d = query.shape
    lib = library()
    need = lib.hif8_paged_attention_workspace_size(tokens, heads, d, max_seq_len)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=query.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if key_cache.stride(0) != key_cache[0].numel() and key_cache.shape[0] > 1:
        check("hif8_paged_attention_strided", lib.hif8_paged_attention_strided(
            _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables), _ptr(seq_lens), _ptr(query_start),
            block_tables.shape[0], tokens, heads, key_cache.shape[2], d, key_cache.shape[0], key_cache.shape[1],
            key_cache.stride(0), block_tables.shape[1], max_seq_len, float(scale), 1 if causal else 0, _ptr(out),
            _ptr(workspace), ws_bytes, _stream(query)))
        return
    check("hif8_paged_attention", lib.hif8_paged_attention(
        _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables), _ptr(seq_lens), _ptr(query_start),
        block_tables.shape[0], tokens, heads, key_cache.shape[2], d, key_cache.shape[0], key_cache.shape[1],
        block_tables.shape[1], max_seq_len, float(scale), 1 if causal else 0, _ptr(out), _ptr(workspace), ws_bytes, _stream(query)))


def paged_attention_noalloc(query, key_cache, value_cache, block_tables, seq_lens, query_start, max_seq_len,
                            scale, out, causal: bool = True) -> None:
    """hif8_paged_attention_noalloc: the split-KV scratch is the library's own
    per-device array, so nothing is allocated for the call."""
    tokens, heads, d = query.shape
    check("hif8_paged_attention_noalloc", library().hif8_paged_attention_noalloc(
        _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables), _ptr(seq_lens), _ptr(query_start),
        block_tables.shape[0], tokens, heads, key_cache.shape[2], d, key_cache.shape[0], key_cache.shape[1],
        block_tables.shape[1], max_seq_len, float(scale), 1 if causal else 0, _ptr(out), _stream(query)))
