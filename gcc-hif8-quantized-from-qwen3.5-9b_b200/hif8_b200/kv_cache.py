"""Paged HiF8 KV cache on the GPU.

Layout contract of the reference (src/vllm_ascend_hif8/kv_cache.py:26-88):
K and V are separate uint8 tensors ``[num_blocks, block_size, kv_heads,
head_size + 4]``; every row is ``head_size`` HiF8 bytes followed by the row's
little-endian FP32 scale (static mode: the layer/head scale of the
checkpoint, repeated for every token).

The write path is one fused kernel (static quant + pack + slot scatter,
replacing kv_runtime._write_hif8_cache, reference kv_runtime.py:1222-1339);
attention reads only the pages each request touches and decodes them in
registers (replacing _gather_dense_hif8 + scaled_decode + the dense attention
call, kv_runtime.py:1375-1563).
"""

from __future__ import annotations

import functools
import json
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

from ._loader import load_ops

HIF8_SCALE_BYTES = 4
HIF8_CACHE_DTYPE = "fp8_per_token_head"
HIF8_METADATA_FILENAME = "hif8_metadata.json"


@dataclass(frozen=True)
class Hif8KVCacheLayout:
    """Physical layout of one HiF8 K/V cache pair (reference kv_cache.py:26-88)."""

    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_size: int
    head_size_v: int | None = None

    def __post_init__(self) -> None:
        values = (self.num_blocks, self.block_size, self.num_kv_heads, self.head_size, self.resolved_head_size_v)
        if any(not isinstance(v, int) or v <= 0 for v in values):
            raise ValueError(f"HIF8 KV dimensions must be positive integers, got {values}")
        if self.head_size % HIF8_SCALE_BYTES:
            raise ValueError("HIF8 KV head_size must be divisible by four so the inline FP32 "
                             f"scale is aligned, got {self.head_size}")
        if self.resolved_head_size_v % HIF8_SCALE_BYTES:
            raise ValueError("HIF8 KV head_size_v must be divisible by four so the inline FP32 "
                             f"scale is aligned, got {self.resolved_head_size_v}")

    @property
    def resolved_head_size_v(self) -> int:
        return self.head_size if self.head_size_v is None else self.head_size_v

    @property
    def key_width(self) -> int:
        return self.head_size + HIF8_SCALE_BYTES

    @property
    def value_width(self) -> int:
        return self.resolved_head_size_v + HIF8_SCALE_BYTES

    @property
    def page_size_bytes(self) -> int:
        return self.block_size * self.num_kv_heads * (self.key_width + self.value_width)

    @property
    def key_page_size_bytes(self) -> int:
        return self.block_size * self.num_kv_heads * self.key_width

    @property
    def value_page_size_bytes(self) -> int:
        return self.block_size * self.num_kv_heads * self.value_width

    def key_shape(self) -> tuple[int, int, int, int]:
        return (self.num_blocks, self.block_size, self.num_kv_heads, self.key_width)

    def value_shape(self) -> tuple[int, int, int, int]:
        return (self.num_blocks, self.block_size, self.num_kv_heads, self.value_width)

    def allocate(self, device):
        """Zero-filled (key_cache, value_cache) on ``device``."""
        import torch

        return (torch.zeros(self.key_shape(), dtype=torch.uint8, device=device),
                torch.zeros(self.value_shape(), dtype=torch.uint8, device=device))


def write_static(key, value, key_cache, value_cache, slot_mapping, key_scale, value_scale, *,
                 num_actual_tokens: int | None = None, validate: bool = False) -> None:
    """Quantise K/V rows with the fixed per-head scales and scatter them into
    their slots.  Negative slots are skipped.  With ``validate=True`` the
    number of slots outside the cache is read back (a host sync) and an
    ``IndexError`` raised, as the reference's write path does
    (kv_runtime.py:1300-1306)."""
    import torch

    load_ops()
    if key.shape[-1] != key_cache.shape[-1] - HIF8_SCALE_BYTES:
        raise ValueError("HIF8 KV input dimensions do not match the cache layout")
    n = key.shape[0] if num_actual_tokens is None else int(num_actual_tokens)
    if n < 0 or n > key.shape[0] or n > value.shape[0]:
        raise ValueError(f"invalid num_actual_tokens={n} for K/V rows {key.shape[0]}/{value.shape[0]}")
    if n == 0:
        return
    slots = slot_mapping[:n]
    if slots.dtype != torch.int64:
        slots = slots.to(torch.int64)
    bad = torch.zeros(1, dtype=torch.int32, device=key.device) if validate else None
    torch.ops.hif8_b200.kv_cache_write(key[:n], value[:n], key_scale.contiguous(), value_scale.contiguous(),
                                       slots.contiguous(), key_cache, value_cache, bad)
    if validate and int(bad.item()) != 0:
        raise IndexError("HIF8 KV slot mapping references an invalid block")


def paged_attention(query, key_cache, value_cache, block_tables, seq_lens: Sequence[int], *,
                    query_lens: Sequence[int] | None = None, scale: float, causal: bool = True):
    """Attention of ``query`` ([tokens, heads, head_size] BF16) over the HiF8
    pages; request b owns the next ``query_lens[b]`` query rows (default 1),
    which sit at the end of its ``seq_lens[b]`` context."""
    import torch

    load_ops()
    lengths = [int(v) for v in seq_lens]
    q_lens = [1] * len(lengths) if query_lens is None else [int(v) for v in query_lens]
    if len(q_lens) != len(lengths) or sum(q_lens) != query.shape[0]:
        raise ValueError("query_lens must describe every query row")
    starts = [0]
    for q in q_lens:
        starts.append(starts[-1] + q)
    dev = query.device
    return torch.ops.hif8_b200.paged_attention(
        query.contiguous(), key_cache, value_cache, block_tables.to(device=dev, dtype=torch.int32).contiguous(),
        torch.tensor(lengths, dtype=torch.int32, device=dev), torch.tensor(starts, dtype=torch.int32, device=dev),
        max(lengths) if lengths else 0, float(scale), bool(causal))


def gather_dense(cache, block_tables, seq_lens: Sequence[int]):
    """Dense BF16 rows ``[sum(seq_lens), heads, head_size]`` of every request,
    grouped by request then token (kv_runtime._gather_dense_hif8 +
    scaled_decode of the reference)."""
    import torch

    load_ops()
    lengths = [int(v) for v in seq_lens]
    starts = [0]
    for n in lengths:
        starts.append(starts[-1] + n)
    dev = cache.device
    return torch.ops.hif8_b200.kv_gather_decode(
        cache, block_tables.to(device=dev, dtype=torch.int32).contiguous(),
        torch.tensor(lengths, dtype=torch.int32, device=dev), torch.tensor(starts, dtype=torch.int32, device=dev),
        starts[-1], max(lengths) if lengths else 0)


@functools.lru_cache(maxsize=8)
def load_static_kv_scales(checkpoint: str) -> dict[int, tuple[tuple[float, ...], tuple[float, ...]]] | None:
    """Per-layer/per-head K and V scales from ``hif8_metadata.json``
    (format of the reference loader, kv_runtime.py:206-266).  Fail-closed: a
    static checkpoint with malformed scale metadata raises ``ValueError``."""
    path = Path(checkpoint) / HIF8_METADATA_FILENAME
    if not path.is_file():
        return None
    metadata = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(metadata, dict):
        raise ValueError(f"invalid HIF8 metadata object: {path}")
    static_checkpoint = metadata.get("format") == "W8A8HIF8_STATIC"
    kv = metadata.get("kv_cache")
    if kv is None:
        if static_checkpoint:
            raise ValueError(f"static HIF8 checkpoint is missing kv_cache metadata: {path}")
        return None
    if not isinstance(kv, dict) or kv.get("mode") != "static_per_layer_per_head":
        raise ValueError(f"unsupported HIF8 kv_cache metadata in {path}")
    layers = kv.get("layers")
    if not isinstance(layers, dict) or not layers:
        raise ValueError(f"HIF8 kv_cache.layers is empty in {path}")
    out: dict[int, tuple[tuple[float, ...], tuple[float, ...]]] = {}
    for raw, entry in layers.items():
        try:
            index = int(raw)
        except (TypeError, ValueError) as error:
            raise ValueError(f"invalid static KV layer index {raw!r}") from error
        if str(index) != str(raw) or index < 0:
            raise ValueError(f"invalid static KV layer index {raw!r}")
        if not isinstance(entry, dict):
            raise ValueError(f"static KV layer {index} is not an object")
        pair = []
        for kind in ("key_scales", "value_scales"):
            raw_scales = entry.get(kind)
            if not isinstance(raw_scales, list) or not raw_scales:
                raise ValueError(f"static KV layer {index} has no {kind}")
            scales = tuple(float(v) for v in raw_scales)
            if any(s <= 0.0 or not math.isfinite(s) for s in scales):
                raise ValueError(f"static KV layer {index} has invalid {kind}")
            pair.append(scales)
        if len(pair[0]) != len(pair[1]):
            raise ValueError(f"static KV layer {index} has different K/V head counts")
        out[index] = (pair[0], pair[1])
    return out
