"""Python face of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The product package (``hif8_b200``) never imports this module.  It is loaded
by ``tests/``, by ``__graft_entry__.smoke()`` as the checker, and by
``bench.py`` for the timed CPU baseline (``--impl reference``).

Byte/integer arithmetic (encode, static quant, scaled decode, KV page write)
lives in the C restatement ``hif8_oracle.c``; floating-point references
(decoded linear, paged attention) are numpy restatements of the reference
plugin's CPU code:

* ``linear``            -> reference ``tests/test_npu_ops.py:296-344`` pattern
                           (decode LUT x scale, then matmul), accumulated in FP64
* ``linear_exact``      -> ``src/vllm_ascend_hif8/reference.py:10-43`` (C, FP64)
* ``paged_attention``   -> ``src/vllm_ascend_hif8/kv_cache.py:314-372`` with the
                           FP32 math of ``tests/test_hif8_kv_npu.py:251-295``
* ``gather_kv_rows``    -> ``src/vllm_ascend_hif8/kv_cache.py:221-252``
* ``embedding``         -> ``src/vllm_ascend_hif8/scheme.py:120-131`` (C decode)
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libhif8_oracle.so"
_lib: ctypes.CDLL | None = None

HIF8_SCALE_BYTES = 4
MAX_FINITE = 32768.0


def build() -> Path:
    """Compile the C oracle in place (``make -C oracle``)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    handle = ctypes.CDLL(str(_LIB_PATH))
    p = ctypes.c_void_p
    i64 = ctypes.c_int64
    handle.hif8o_encode_value.argtypes = [ctypes.c_float]
    handle.hif8o_encode_value.restype = ctypes.c_uint8
    handle.hif8o_decode_bf16_bits.argtypes = [ctypes.c_uint8]
    handle.hif8o_decode_bf16_bits.restype = ctypes.c_uint16
    handle.hif8o_decode_table.argtypes = [p]
    handle.hif8o_encode_lut4096.argtypes = [p]
    handle.hif8o_encode_tensor.argtypes = [p, i64, p]
    handle.hif8o_static_quant.argtypes = [p, ctypes.c_int, i64, i64, p, i64, p, p]
    handle.hif8o_dynamic_quant.argtypes = [p, ctypes.c_int, i64, i64, p, p]
    handle.hif8o_scaled_decode.argtypes = [p, i64, i64, i64, p, p]
    handle.hif8o_kv_write.argtypes = [p, ctypes.c_int, i64, i64, i64, p, p, p, i64, i64]
    handle.hif8o_kv_write.restype = i64
    handle.hif8o_linear_f64.argtypes = [p, p, p, p, p, i64, i64, i64, p]
    handle.hif8o_f32_to_bf16_bits.argtypes = [ctypes.c_float]
    handle.hif8o_f32_to_bf16_bits.restype = ctypes.c_uint16
    _lib = handle
    return handle


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


# ----------------------------------------------------------------- codec ---

def decode_table() -> np.ndarray:
    out = np.empty(256, dtype=np.float32)
    lib().hif8o_decode_table(_ptr(out))
    return out


def decode_bf16_table() -> np.ndarray:
    handle = lib()
    return np.array([handle.hif8o_decode_bf16_bits(b) for b in range(256)], dtype=np.uint16)


def encode_lut4096() -> np.ndarray:
    out = np.empty(4096, dtype=np.uint8)
    lib().hif8o_encode_lut4096(_ptr(out))
    return out


def encode_value(value: float) -> int:
    return int(lib().hif8o_encode_value(float(value)))


def encode_tensor(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().hif8o_encode_tensor(_ptr(x), x.size, _ptr(out))
    return out


# --------------------------------------------------------- half helpers ---

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Nearest-even BF16 bits; NaN -> 0x7FC0 (c10::BFloat16 rule)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), rounded)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---------------------------------------------------------- static quant ---

def static_quant(x_bits: np.ndarray, scale: np.ndarray, *, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """HiF8 bytes + per-row scale for a [..., K] FP16/BF16 bit tensor.

    ``scale`` has S entries, S divides the row count; row r uses scale[r % S]
    (the kernel contract of ``hif8_static_quant``, reference
    csrc/opp/op_kernel/hif8_static_quant.cpp and native.py:90-124).
    """
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    scale = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    k = x_bits.shape[-1]
    rows = x_bits.size // k if k else 0
    out = np.empty(x_bits.shape, dtype=np.uint8)
    row_scale = np.empty(rows, dtype=np.float32)
    lib().hif8o_static_quant(_ptr(x_bits), 1 if dtype == "bf16" else 0, rows, k, _ptr(scale),
                             scale.size, _ptr(out), _ptr(row_scale))
    return out, row_scale


def dynamic_quant(x_bits: np.ndarray, *, dtype: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """HiF8 bytes + per-row scale of the dynamic quant (reference
    codec.py:205-255, choose_row_scale + quantize_rows; the contract of op
    hif8_dynamic_quant, csrc/opp/op_kernel/hif8_dynamic_quant.cpp): scale =
    max(amax of the row's finite |x|, 1e-12), codes of x / scale."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    k = x_bits.shape[-1]
    rows = x_bits.size // k if k else 0
    out = np.empty(x_bits.shape, dtype=np.uint8)
    row_scale = np.empty(rows, dtype=np.float32)
    lib().hif8o_dynamic_quant(_ptr(x_bits), 1 if dtype == "bf16" else 0, rows, k, _ptr(out), _ptr(row_scale))
    return out, row_scale


def scaled_decode(data: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """BF16 bits of decode(data[r, k]) * scale[r]."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    rows, k = data.shape
    out = np.empty((rows, k), dtype=np.uint16)
    lib().hif8o_scaled_decode(_ptr(data), rows, k, k, _ptr(scale), _ptr(out))
    return out


def embedding(codes: np.ndarray, scale: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """BF16 bits [*ids.shape, hidden] of the HiF8 token-embedding lookup
    (reference src/vllm_ascend_hif8/scheme.py:120-131): decode of the
    gathered rows times the row scale rounded to BF16, one BF16 rounding of
    the (exact) FP32 product -- i.e. scaled_decode with BF16-rounded scales.
    NaN codes give the canonical 0x7FC0 (the reference's CPU run writes
    0xFFFF through ATen's vectorised BF16 cast: the same value).  Ids outside
    [0, vocab) give zero rows."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    vocab, hidden = codes.shape
    scale = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    ok = (flat >= 0) & (flat < vocab)
    safe = np.where(ok, flat, 0)
    out = scaled_decode(codes[safe], round_bf16(scale[safe]))
    out[~ok] = 0
    return out.reshape(*np.shape(ids), hidden)


# ------------------------------------------------------------------- KV ---

def pack_kv_rows(data: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """[tokens, heads, D] bytes + [tokens, heads] FP32 -> [tokens, heads, D+4]
    (reference kv_cache.py:151-170)."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    packed = np.empty((*data.shape[:-1], data.shape[-1] + HIF8_SCALE_BYTES), dtype=np.uint8)
    packed[..., :-HIF8_SCALE_BYTES] = data
    packed[..., -HIF8_SCALE_BYTES:] = scale.view(np.uint8).reshape(*scale.shape, HIF8_SCALE_BYTES)
    return packed


def unpack_kv_rows(packed: np.ndarray, head_size: int) -> tuple[np.ndarray, np.ndarray]:
    data = packed[..., :head_size]
    scale = np.ascontiguousarray(packed[..., head_size:]).view(np.float32).reshape(packed.shape[:-1])
    return data, scale


def kv_write(src_bits: np.ndarray, head_scale: np.ndarray, slot_mapping: np.ndarray, cache: np.ndarray,
             *, dtype: str = "bf16") -> int:
    """In-place fused static quant + pack + slot scatter into ``cache``."""
    src_bits = np.ascontiguousarray(src_bits, dtype=np.uint16)
    head_scale = np.ascontiguousarray(head_scale, dtype=np.float32)
    slots = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    assert cache.flags["C_CONTIGUOUS"] and cache.dtype == np.uint8
    tokens, heads, head_size = src_bits.shape
    return int(lib().hif8o_kv_write(_ptr(src_bits), 1 if dtype == "bf16" else 0, tokens, heads, head_size,
                                    _ptr(head_scale), _ptr(slots), _ptr(cache), cache.shape[0], cache.shape[1]))


def gather_kv_rows(cache: np.ndarray, block_table: np.ndarray, length: int, block_size: int) -> np.ndarray:
    blocks = (length + block_size - 1) // block_size
    rows = cache[np.asarray(block_table[:blocks], dtype=np.int64)].reshape(-1, *cache.shape[2:])
    return rows[:length]


def paged_attention(query: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray,
                    block_table: np.ndarray, seq_lens, *, block_size: int, scale: float,
                    query_lens=None, causal: bool = True, bf16_kv: bool = True) -> np.ndarray:
    """FP32 GQA paged attention over decoded HiF8 pages.

    K/V rows are decoded as ``decode(byte) * row_scale`` and, with
    ``bf16_kv``, rounded to BF16 exactly as the reference's scaled_decode
    path materialises them before attention.  Query rows of a request are its
    last ``q_len`` positions (right-aligned causal mask).
    """
    query = np.asarray(query, dtype=np.float32)
    lut = decode_table()
    head_size = key_cache.shape[-1] - HIF8_SCALE_BYTES
    head_size_v = value_cache.shape[-1] - HIF8_SCALE_BYTES
    kv_heads = key_cache.shape[2]
    num_heads = query.shape[1]
    group = num_heads // kv_heads
    lengths = [int(v) for v in seq_lens]
    q_lengths = [1] * len(lengths) if query_lens is None else [int(v) for v in query_lens]
    outputs = []
    q_begin = 0
    for request, (length, q_len) in enumerate(zip(lengths, q_lengths)):
        k_rows = gather_kv_rows(key_cache, block_table[request], length, block_size)
        v_rows = gather_kv_rows(value_cache, block_table[request], length, block_size)
        k_data, k_scale = unpack_kv_rows(k_rows, head_size)
        v_data, v_scale = unpack_kv_rows(v_rows, head_size_v)
        keys = lut[k_data] * k_scale[..., None]
        values = lut[v_data] * v_scale[..., None]
        if bf16_kv:
            keys, values = round_bf16(keys), round_bf16(values)
        keys = np.repeat(keys, group, axis=1).astype(np.float64)
        values = np.repeat(values, group, axis=1).astype(np.float64)
        q = query[q_begin:q_begin + q_len].astype(np.float64)
        q_begin += q_len
        logits = np.einsum("qhd,khd->qhk", q, keys) * float(scale)
        if causal:
            positions = np.arange(q_len) + length - q_len
            mask = np.arange(length)[None, None, :] > positions[:, None, None]
            logits = np.where(mask, -np.inf, logits)
        logits = logits - logits.max(axis=-1, keepdims=True)
        probs = np.exp(logits)
        probs /= probs.sum(axis=-1, keepdims=True)
        outputs.append(np.einsum("qhk,khd->qhd", probs, values).astype(np.float32))
    if not outputs:
        return np.empty((0, num_heads, head_size_v), dtype=np.float32)
    return np.concatenate(outputs, axis=0)


# --------------------------------------------------------------- linear ---

def linear(a: np.ndarray, w: np.ndarray, token_scale: np.ndarray, channel_scale: np.ndarray,
           bias: np.ndarray | None = None) -> np.ndarray:
    """(decode(a) x ts) @ (decode(w) x cs)^T (+ bias), accumulated in FP64."""
    lut = decode_table().astype(np.float64)
    a_dec = lut[np.asarray(a, dtype=np.uint8)]
    w_dec = lut[np.asarray(w, dtype=np.uint8)]
    acc = a_dec @ w_dec.T
    out = acc * np.asarray(token_scale, dtype=np.float64).reshape(-1, 1) \
        * np.asarray(channel_scale, dtype=np.float64).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float64).reshape(1, -1)
    return out


def linear_f32(a: np.ndarray, w: np.ndarray, token_scale: np.ndarray, channel_scale: np.ndarray,
               bias: np.ndarray | None = None) -> np.ndarray:
    """The reference's CPU linear in FP32 (decode LUT, scale, matmul): the
    timed CPU baseline path (tests/test_npu_ops.py:334-336 of the reference)."""
    lut = decode_table()
    a_dec = lut[a] * np.asarray(token_scale, dtype=np.float32).reshape(-1, 1)
    w_dec = lut[w] * np.asarray(channel_scale, dtype=np.float32).reshape(-1, 1)
    out = a_dec @ w_dec.T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float32).reshape(1, -1)
    return out


def linear_exact(a: np.ndarray, w: np.ndarray, token_scale: np.ndarray, channel_scale: np.ndarray,
                 bias: np.ndarray | None = None) -> np.ndarray:
    """reference.linear_u8_u8 restated in C (FP64 loops); small shapes only."""
    a = np.ascontiguousarray(a, dtype=np.uint8)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    ts = np.ascontiguousarray(token_scale, dtype=np.float32).reshape(-1)
    cs = np.ascontiguousarray(channel_scale, dtype=np.float32).reshape(-1)
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    lib().hif8o_linear_f64(_ptr(a), _ptr(w), _ptr(ts), _ptr(cs), None if b is None else _ptr(b), m, n, k, _ptr(out))
    return out


# ------------------------------------------------- synthetic input makers ---

def quantize_rows_amax(w: np.ndarray, scale_factor: float = MAX_FINITE) -> tuple[np.ndarray, np.ndarray]:
    """Per-row amax weight quantisation (torch_codec.quantize_tensor_rows,
    reference torch_codec.py:52-73): scale = max(row amax, 1e-12) / factor."""
    w32 = np.asarray(w, dtype=np.float32)
    amax = np.abs(w32).max(axis=-1)
    scale = (np.maximum(amax, np.float32(1.0e-12)) / np.float32(scale_factor)).astype(np.float32)
    q = (w32 / scale[..., None]).astype(np.float32)
    return encode_tensor(q), scale


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
