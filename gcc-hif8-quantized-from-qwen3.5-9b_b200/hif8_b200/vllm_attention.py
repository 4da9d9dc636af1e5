"""vLLM (CUDA) attention backend for the physical HiF8 KV cache.

The reference routes vLLM-Ascend's attention through a HiF8 cache adapter
(src/vllm_ascend_hif8/kv_runtime.py): K/V rows are quantised and packed into
uint8 pages on write (``_write_hif8_cache``, kv_runtime.py:1222-1339), and
attention reads the pages back (``_forward_hif8_attention``,
kv_runtime.py:1470-1563), enabled per process by ``HIF8_KV_CACHE=1`` and
``install_hif8_kv_cache_adapter`` (kv_runtime.py:1655-1667).  On CUDA vLLM the
same cache is an attention backend registered as ``CUSTOM``:

* the cache dtype is vLLM's ``fp8_per_token_head``, whose page budget (one
  byte per element plus one FP32 scale per token and head, K and V) is
  exactly the HiF8 page: every row is head_size HiF8 codes followed by the
  row's FP32 scale.  ``Hif8AttentionBackend.get_kv_cache_shape`` lays a
  block out as vLLM's block-major page ``[num_blocks, 2, block_size,
  kv_heads, head_size + 4]`` (K rows, then V rows), which the kernels read
  with a block stride, so hybrid models whose pages vLLM pads keep working;
* ``do_kv_cache_update`` quantises the step's K/V rows with the checkpoint's
  static per-layer, per-head scales and scatters them into their slots in one
  kernel (``hif8_b200::kv_cache_write``); a checkpoint without KV scales (the
  legacy dynamic format) gets per-row dynamic scales
  (``hif8_dynamic_quant``), as the reference's ``_quantize_kv`` does;
* ``forward`` runs paged attention over the pages each request touches
  (``hif8_b200::paged_attention``): one query row per request takes the
  split-KV tensor-core decode kernel, prefill and mixed (chunked-prefill)
  batches the multi-row kernel, both with the right-aligned causal mask of
  vLLM's query layout.

Activation: ``install_hif8_kv_cache_adapter()`` (a no-op unless
``HIF8_KV_CACHE=1``; ``vllm_adapter.register()`` calls it) registers the
backend as ``CUSTOM`` and makes new ``CacheConfig`` / ``AttentionConfig``
objects default to ``fp8_per_token_head`` and that backend, so an engine
started with the variable set serves its full-attention layers from HiF8
pages (the gated-delta-net layers keep vLLM's state caches).
"""

from __future__ import annotations

import functools
import inspect
import os
import re
from dataclasses import dataclass
from typing import Any, ClassVar

import torch
from vllm.v1.attention.backend import (
    AttentionBackend,
    AttentionCGSupport,
    AttentionImpl,
    AttentionMetadata,
    AttentionMetadataBuilder,
    AttentionType,
    CommonAttentionMetadata,
)

from . import kv_cache as hif8_kv
from . import native
from ._loader import load_ops

HIF8_KV_CACHE_ENV = "HIF8_KV_CACHE"
HIF8_KV_CACHE_DTYPE = hif8_kv.HIF8_CACHE_DTYPE  # "fp8_per_token_head"
HIF8_SCALE_BYTES = hif8_kv.HIF8_SCALE_BYTES
BACKEND_NAME = "CUSTOM"
_LAYER_INDEX = re.compile(r"(?:^|\.)layers\.(\d+)(?=\.|$)")


def hif8_kv_cache_enabled() -> bool:
    """Whether the physical HiF8 KV cache is enabled for this process
    (reference kv_runtime.py:176-179)."""
    return os.environ.get(HIF8_KV_CACHE_ENV) == "1"


def attention_layer_index(layer_name: str) -> int:
    """Decoder layer index of an attention prefix ``...layers.<i>...``
    (reference kv_runtime.py:182-191)."""
    found = _LAYER_INDEX.findall(str(layer_name))
    if len(found) != 1:
        raise ValueError(f"cannot resolve one decoder layer index from HIF8 attention prefix {layer_name!r}")
    return int(found[0])


def _checkpoint_path(vllm_config: Any) -> str | None:
    """The checkpoint directory of an engine config (reference
    kv_runtime.py:194-203), or None when there is no model config."""
    model_config = getattr(vllm_config, "model_config", None)
    if model_config is None:
        return None
    path = getattr(model_config, "model_weights", "") or getattr(model_config, "model", "")
    return str(path) if path else None


def checkpoint_kv_scales(vllm_config: Any) -> dict[int, tuple[tuple[float, ...], tuple[float, ...]]] | None:
    """Static K/V scales of the engine's checkpoint (``hif8_metadata.json``),
    None for a checkpoint without them (legacy dynamic KV)."""
    path = _checkpoint_path(vllm_config)
    if path is None or not os.path.isdir(path):
        return None
    return hif8_kv.load_static_kv_scales(path)


def rank_head_scales(values: tuple[float, ...], local_heads: int, tp_size: int = 1,
                     tp_rank: int = 0) -> tuple[float, ...]:
    """The scales of this rank's KV heads.  A checkpoint stores one scale
    per KV head of the whole model; vLLM's QKV projection gives rank r heads
    [r*H, (r+1)*H) when the heads divide over the ranks, and the single head
    r // (tp / heads) when there are fewer heads than ranks."""
    total = len(values)
    if total == local_heads:
        return tuple(values)
    if tp_size > 1 and total % tp_size == 0 and total // tp_size == local_heads:
        return tuple(values[tp_rank * local_heads:(tp_rank + 1) * local_heads])
    if tp_size > 1 and total < tp_size and tp_size % total == 0 and local_heads == 1:
        return (values[tp_rank // (tp_size // total)],)
    raise ValueError(f"static HIF8 KV scales: {total} scales for {local_heads} heads on rank {tp_rank} "
                     f"of {tp_size}")


def _tp_world() -> tuple[int, int]:
    try:
        from vllm.distributed import get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size

        return get_tensor_model_parallel_world_size(), get_tensor_model_parallel_rank()
    except (AssertionError, RuntimeError):
        return 1, 0


def cache_planes(kv_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V planes ``[num_blocks, block_size, kv_heads, head_size + 4]``
    of a block-major cache ``[num_blocks, 2, block_size, kv_heads, width]``
    (each plane's blocks one page apart; reference kv_runtime.py:533-571)."""
    if kv_cache.ndim != 5 or kv_cache.shape[1] != 2 or kv_cache.dtype != torch.uint8:
        raise ValueError("HIF8 KV cache must be uint8 [num_blocks, 2, block_size, kv_heads, head_size + 4], "
                         f"got {tuple(kv_cache.shape)} {kv_cache.dtype}")
    return kv_cache[:, 0], kv_cache[:, 1]


# ------------------------------------------------------------- metadata ---

@dataclass
class Hif8AttentionMetadata(AttentionMetadata):
    """One step's batch as the HiF8 kernels read it: request r owns query
    rows [query_start_loc[r], query_start_loc[r+1]), which are the last rows
    of its seq_lens[r]-token context (reference kv_runtime.py:588-641)."""

    num_actual_tokens: int
    num_reqs: int
    max_query_len: int
    max_seq_len: int
    query_start_loc: torch.Tensor  # int32 [num_reqs + 1]
    seq_lens: torch.Tensor         # int32 [num_reqs]
    block_table: torch.Tensor      # int32 [num_reqs, max_blocks]
    slot_mapping: torch.Tensor     # int64 [num_actual_tokens]
    causal: bool = True


class Hif8AttentionMetadataBuilder(AttentionMetadataBuilder[Hif8AttentionMetadata]):
    """Views of vLLM's common per-step metadata; nothing is copied.  The
    kernels take the batch size and the longest context from the host, so
    attention runs outside captured CUDA graphs (vLLM then captures the rest
    of the step piecewise)."""

    _cudagraph_support: ClassVar[AttentionCGSupport] = AttentionCGSupport.NEVER

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> Hif8AttentionMetadata:
        m = common_attn_metadata
        n = int(m.num_reqs)
        return Hif8AttentionMetadata(
            num_actual_tokens=int(m.num_actual_tokens), num_reqs=n, max_query_len=int(m.max_query_len),
            max_seq_len=int(m.max_seq_len), query_start_loc=m.query_start_loc[:n + 1], seq_lens=m.seq_lens[:n],
            block_table=m.block_table_tensor[:n], slot_mapping=m.slot_mapping, causal=bool(m.causal))


# -------------------------------------------------------------- backend ---

class Hif8AttentionBackend(AttentionBackend):
    """Attention over the physical HiF8 KV cache (registered as ``CUSTOM``)."""

    accept_output_buffer: bool = True
    forward_includes_kv_cache_update: bool = False
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.bfloat16]
    supported_kv_cache_dtypes: ClassVar[list[str]] = [HIF8_KV_CACHE_DTYPE]

    @staticmethod
    def get_name() -> str:
        return BACKEND_NAME

    @staticmethod
    def get_impl_cls() -> type["Hif8AttentionImpl"]:
        return Hif8AttentionImpl

    @staticmethod
    def get_builder_cls() -> type[Hif8AttentionMetadataBuilder]:
        return Hif8AttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        # vLLM budgets fp8_per_token_head pages as one byte per element plus
        # one FP32 scale per (token, head) for K and for V: the HiF8 rows
        if cache_dtype_str != HIF8_KV_CACHE_DTYPE:
            raise ValueError(f"the HiF8 KV cache needs kv_cache_dtype={HIF8_KV_CACHE_DTYPE!r}, "
                             f"got {cache_dtype_str!r}")
        return (num_blocks, 2, block_size, num_kv_heads, head_size + HIF8_SCALE_BYTES)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        if include_num_layers_dimension:
            raise NotImplementedError("the HiF8 KV cache has no cross-layer layout")
        return (0, 1, 2, 3, 4)

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size % HIF8_SCALE_BYTES == 0 and 0 < head_size <= 1024

    @classmethod
    def supports_compute_capability(cls, capability) -> bool:
        return capability.major == 10

    @classmethod
    def supports_block_size(cls, block_size: int | None) -> bool:
        return block_size is None or block_size > 0


# ----------------------------------------------------------------- impl ---

class Hif8AttentionImpl(AttentionImpl[Hif8AttentionMetadata]):
    """K/V writes into HiF8 pages and attention over them for one layer
    (reference kv_runtime.py:1222-1339 write, 1470-1563 attention)."""

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes: list[float] | None = None, sliding_window: int | None = None,
                 kv_cache_dtype: str = "auto", logits_soft_cap: float | None = None,
                 attn_type: str = AttentionType.DECODER, kv_sharing_target_layer_name: str | None = None,
                 **extra: Any) -> None:
        if alibi_slopes is not None:
            raise NotImplementedError("HIF8 attention does not support ALiBi")
        if sliding_window is not None:
            raise NotImplementedError("HIF8 attention does not support sliding windows")
        if logits_soft_cap:
            raise NotImplementedError("HIF8 attention does not support logit soft-capping")
        if extra.get("sinks") is not None:
            raise NotImplementedError("HIF8 attention does not support attention sinks")
        if attn_type != AttentionType.DECODER:
            raise NotImplementedError(f"HIF8 attention serves decoder attention only, got {attn_type}")
        if kv_cache_dtype != HIF8_KV_CACHE_DTYPE:
            raise ValueError(f"HIF8 attention needs kv_cache_dtype={HIF8_KV_CACHE_DTYPE!r}, got {kv_cache_dtype!r}")
        self.num_heads = int(num_heads)
        self.head_size = int(head_size)
        self.scale = float(scale)
        self.num_kv_heads = int(num_kv_heads or num_heads)
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.kv_cache_dtype = kv_cache_dtype
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self._explicit_scales: tuple[tuple[float, ...], tuple[float, ...]] | None = None
        self._scale_tensors: tuple[torch.Tensor, torch.Tensor] | None = None
        try:
            from vllm.config import get_current_vllm_config

            self._checkpoint_scales = checkpoint_kv_scales(get_current_vllm_config())
        except (AssertionError, RuntimeError):
            self._checkpoint_scales = None
        load_ops()  # fail loudly now, not at the first step, without the kernels

    # ---- scales ----------------------------------------------------------
    def set_static_kv_scales(self, key_scales, value_scales) -> None:
        """Bind this layer's per-head K/V scales (this rank's heads)
        instead of the checkpoint's ``hif8_metadata.json``."""
        k = tuple(float(v) for v in key_scales)
        v = tuple(float(x) for x in value_scales)
        if len(k) != self.num_kv_heads or len(v) != self.num_kv_heads:
            raise ValueError(f"expected {self.num_kv_heads} K and V scales, got {len(k)} and {len(v)}")
        self._explicit_scales = (k, v)
        self._scale_tensors = None

    def static_kv_scales(self, layer: Any, device: torch.device) -> tuple[torch.Tensor, torch.Tensor] | None:
        """FP32 per-head K and V scales of this layer on ``device``, or None
        when the checkpoint has no static KV scales (dynamic rows).  A
        checkpoint with scales but none for this layer is an error
        (fail-closed, reference kv_runtime.py:1136-1160)."""
        if self._scale_tensors is not None and self._scale_tensors[0].device == device:
            return self._scale_tensors
        values = self._explicit_scales
        if values is None:
            if self._checkpoint_scales is None:
                return None
            index = attention_layer_index(getattr(layer, "layer_name", ""))
            if index not in self._checkpoint_scales:
                raise ValueError(f"static HIF8 checkpoint has no KV scales for attention layer {index} "
                                 f"({getattr(layer, 'layer_name', '')})")
            k, v = self._checkpoint_scales[index]
            tp_size, tp_rank = _tp_world()
            values = (rank_head_scales(k, self.num_kv_heads, tp_size, tp_rank),
                      rank_head_scales(v, self.num_kv_heads, tp_size, tp_rank))
        self._scale_tensors = tuple(torch.tensor(s, dtype=torch.float32, device=device) for s in values)
        return self._scale_tensors

    # ---- cache write -----------------------------------------------------
    def do_kv_cache_update(self, layer: Any, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
        """Quantise and scatter the step's K/V rows; negative slots (padding)
        are skipped (reference kv_runtime.py:1222-1339)."""
        if self.kv_sharing_target_layer_name is not None:
            return  # the producer layer writes the shared cache
        if key.shape[-1] != self.head_size or value.shape[-1] != self.head_size:
            raise ValueError(f"HIF8 KV input dimensions do not match the layer: K={key.shape[-1]}, "
                             f"V={value.shape[-1]}, head_size={self.head_size}")
        n = min(int(key.shape[0]), int(slot_mapping.shape[0]))
        if n == 0:
            return
        key_cache, value_cache = cache_planes(kv_cache)
        slots = slot_mapping[:n]
        if slots.dtype != torch.int64:
            slots = slots.to(torch.int64)
        scales = self.static_kv_scales(layer, key.device)
        if scales is None:
            self._write_dynamic(key[:n], value[:n], slots, key_cache, value_cache)
            return
        torch.ops.hif8_b200.kv_cache_write(key[:n], value[:n], scales[0], scales[1], slots, key_cache,
                                           value_cache, None)

    @staticmethod
    def _write_dynamic(key, value, slots, key_cache, value_cache) -> None:
        """Legacy checkpoints: each (token, head) row gets its own dynamic
        scale (``hif8_dynamic_quant``), packed after its codes and copied
        into the slot (reference kv_runtime.py:1168-1199, 1281-1299)."""
        valid = slots >= 0
        if not bool(valid.any()):
            return
        block_size = key_cache.shape[1]
        blocks, offsets = slots[valid] // block_size, slots[valid] % block_size
        if bool((blocks >= key_cache.shape[0]).any()):
            raise IndexError("HIF8 KV slot mapping references an invalid block")
        for src, plane in ((key, key_cache), (value, value_cache)):
            n, heads, d = src.shape
            codes, scale = native.dynamic_quant(src.reshape(n * heads, d))
            rows = torch.cat([codes.reshape(n, heads, d),
                              scale.contiguous().view(torch.uint8).reshape(n, heads, HIF8_SCALE_BYTES)], dim=-1)
            plane[blocks, offsets] = rows[valid]

    # ---- attention -------------------------------------------------------
    def forward(self, layer: Any, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: torch.Tensor, attn_metadata: Hif8AttentionMetadata | None,
                output: torch.Tensor | None = None, output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        """Attention of the step's query rows over their requests' pages
        (the rows were written by ``do_kv_cache_update`` first); rows past
        the batch's real tokens are zero (reference kv_runtime.py:1470-1563)."""
        if output is None:
            raise ValueError("HIF8 attention requires an output buffer")
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("HIF8 attention does not support output quantization")
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        n = attn_metadata.num_actual_tokens
        if n > 0:
            key_cache, value_cache = cache_planes(kv_cache)
            q = query[:n]
            if not q.is_contiguous() or q.storage_offset() != 0:
                q = q.contiguous()
            out = torch.ops.hif8_b200.paged_attention(
                q, key_cache, value_cache, attn_metadata.block_table, attn_metadata.seq_lens,
                attn_metadata.query_start_loc, attn_metadata.max_seq_len, self.scale, attn_metadata.causal)
            output[:n].copy_(out.view(output[:n].shape))
        if n < output.shape[0]:
            output[n:].zero_()
        return output


# ------------------------------------------------------------- install ---

_installed = False
_originals: dict[str, Any] = {}


def _force_config_field(cls: type, key: str, field: str, value: Any, accepted: tuple[Any, ...],
                        flag: str) -> None:
    """Wrap ``cls.__init__`` so that, with the HiF8 KV cache enabled,
    ``field`` becomes ``value`` when the caller left it at one of
    ``accepted`` and the construction fails otherwise."""
    original = cls.__init__
    if getattr(original, "_hif8_kv_adapter", False):
        return
    signature = inspect.signature(cls)

    @functools.wraps(original)
    def init(self, *args, **kwargs):
        if not hif8_kv_cache_enabled():
            return original(self, *args, **kwargs)
        bound = signature.bind(*args, **kwargs)
        requested = bound.arguments.get(field, accepted[0])
        if requested not in accepted and requested != value:
            raise ValueError(f"{HIF8_KV_CACHE_ENV}=1 requires {flag}, got {requested!r}")
        bound.arguments[field] = value
        original(self, **bound.arguments)

    init._hif8_kv_adapter = True
    _originals[key] = (cls, original)
    cls.__init__ = init


def install_hif8_kv_cache_adapter() -> None:
    """With ``HIF8_KV_CACHE=1``: register ``Hif8AttentionBackend`` as vLLM's
    ``CUSTOM`` attention backend and make new ``CacheConfig`` /
    ``AttentionConfig`` objects select the HiF8 cache dtype and that backend
    (an explicit other choice is refused).  Idempotent; a no-op without the
    variable (reference kv_runtime.py:1655-1667)."""
    global _installed
    if _installed or not hif8_kv_cache_enabled():
        return
    from vllm.config.attention import AttentionConfig
    from vllm.config.cache import CacheConfig
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.CUSTOM, f"{Hif8AttentionBackend.__module__}.Hif8AttentionBackend")
    _force_config_field(CacheConfig, "CacheConfig.__init__", "cache_dtype", HIF8_KV_CACHE_DTYPE, ("auto",),
                        f"kv_cache_dtype={HIF8_KV_CACHE_DTYPE} or auto")
    _force_config_field(AttentionConfig, "AttentionConfig.__init__", "backend", AttentionBackendEnum.CUSTOM,
                        (None, "auto", "AUTO", "CUSTOM", "custom"), "attention backend CUSTOM or auto")
    _installed = True


def reset_hif8_kv_cache_adapter_for_tests() -> None:
    """Undo ``install_hif8_kv_cache_adapter`` (isolated tests; reference
    kv_runtime.py:1670-1706)."""
    global _installed
    for cls, original in _originals.values():
        cls.__init__ = original
    _originals.clear()
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum

        AttentionBackendEnum.CUSTOM.clear_override()
    except (AttributeError, ImportError):
        pass
    hif8_kv.load_static_kv_scales.cache_clear()
    _installed = False
