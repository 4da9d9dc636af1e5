"""Checks of the vLLM attention backend for the HiF8 KV cache
(hif8_b200.vllm_attention) on vLLM's own ``Attention`` layer, run as a child
process by tests/test_vllm_attention_cpu.py (mode ``cpu``: registration, the
config hooks, cache shapes and page budget, metadata, refusals) and
tests/test_vllm_attention_gpu.py (mode ``gpu``: cache writes and attention
through ``Attention.forward`` against the oracle).  Exits non-zero on the
first failed check."""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "gcc-hif8-quantized-from-qwen3.5-9b_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

HEADS, KV_HEADS, D, BS, NUM_BLOCKS = 8, 2, 256, 16, 40
DTYPE = "fp8_per_token_head"
PREFIX = "language_model.model.layers.{}.self_attn.attn"


def _expect_raises(exc, fn, match):
    try:
        fn()
    except exc as e:
        assert match in str(e), f"expected {match!r} in {e!r}"
        return
    raise AssertionError(f"expected {exc.__name__} ({match})")


def _config_hooks(va):
    from vllm.config.attention import AttentionConfig
    from vllm.config.cache import CacheConfig
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    os.environ.pop(va.HIF8_KV_CACHE_ENV, None)
    va.install_hif8_kv_cache_adapter()  # disabled: nothing changes
    assert CacheConfig().cache_dtype == "auto" and AttentionConfig().backend is None
    os.environ[va.HIF8_KV_CACHE_ENV] = "1"
    va.install_hif8_kv_cache_adapter()
    va.install_hif8_kv_cache_adapter()  # idempotent
    assert AttentionBackendEnum.CUSTOM.get_class() is va.Hif8AttentionBackend
    assert CacheConfig().cache_dtype == DTYPE and CacheConfig(cache_dtype="auto").cache_dtype == DTYPE
    assert CacheConfig(block_size=32).block_size == 32
    assert AttentionConfig().backend == AttentionBackendEnum.CUSTOM
    assert AttentionConfig(backend="auto").backend == AttentionBackendEnum.CUSTOM
    _expect_raises(ValueError, lambda: CacheConfig(cache_dtype="bfloat16"), "kv_cache_dtype")
    _expect_raises(ValueError, lambda: AttentionConfig(backend="FLASH_ATTN"), "attention backend")
    va.reset_hif8_kv_cache_adapter_for_tests()
    os.environ.pop(va.HIF8_KV_CACHE_ENV, None)
    assert CacheConfig().cache_dtype == "auto" and AttentionConfig().backend is None


def _host_rules(va):
    assert va.attention_layer_index("language_model.model.layers.11.self_attn.attn") == 11
    assert va.attention_layer_index("layers.0.attn") == 0
    _expect_raises(ValueError, lambda: va.attention_layer_index("model.norm"), "layer index")
    assert va.rank_head_scales((1.0, 2.0), 2) == (1.0, 2.0)
    assert va.rank_head_scales((1.0, 2.0, 3.0, 4.0), 2, tp_size=2, tp_rank=1) == (3.0, 4.0)
    assert va.rank_head_scales((1.0, 2.0), 1, tp_size=4, tp_rank=3) == (2.0,)  # heads replicated over ranks
    _expect_raises(ValueError, lambda: va.rank_head_scales((1.0, 2.0, 3.0), 2, tp_size=2), "scales")
    shape = va.Hif8AttentionBackend.get_kv_cache_shape(7, BS, KV_HEADS, D, DTYPE)
    assert shape == (7, 2, BS, KV_HEADS, D + 4)
    assert va.Hif8AttentionBackend.get_kv_cache_block_dim(BS, KV_HEADS, D, DTYPE) == 0
    _expect_raises(ValueError, lambda: va.Hif8AttentionBackend.get_kv_cache_shape(7, BS, KV_HEADS, D, "auto"),
                   "kv_cache_dtype")
    assert va.Hif8AttentionBackend.supports_head_size(256) and not va.Hif8AttentionBackend.supports_head_size(66)


def _layer(va, index, cache_dtype=DTYPE, **extra):
    from vllm.config.cache import CacheConfig
    from vllm.model_executor.layers.attention import Attention

    return Attention(HEADS, D, 1.0 / math.sqrt(D), num_kv_heads=KV_HEADS,
                     cache_config=CacheConfig(cache_dtype=cache_dtype, block_size=BS), prefix=PREFIX.format(index),
                     attn_backend=va.Hif8AttentionBackend, **extra)


def _layer_contract(va, vllm_config):
    attn = _layer(va, 3)
    assert isinstance(attn.impl, va.Hif8AttentionImpl) and attn.impl.kv_cache_dtype == DTYPE
    spec = attn.get_kv_cache_spec(vllm_config)
    # vLLM's page budget for fp8_per_token_head is exactly one HiF8 page
    assert spec.page_size_bytes == 2 * BS * KV_HEADS * (D + 4), spec.page_size_bytes
    assert spec.dtype == torch.uint8
    _expect_raises(NotImplementedError, lambda: _layer(va, 4, per_layer_sliding_window=128), "sliding")
    _expect_raises(ValueError, lambda: _layer(va, 5, cache_dtype="auto"), "kv_cache_dtype")
    # without a checkpoint there are no static scales: dynamic rows
    assert attn.impl.static_kv_scales(attn, torch.device("cpu")) is None
    attn.impl.set_static_kv_scales([0.5, 0.25], [0.125, 1.0])
    ks, vs = attn.impl.static_kv_scales(attn, torch.device("cpu"))
    assert ks.tolist() == [0.5, 0.25] and vs.tolist() == [0.125, 1.0]
    _expect_raises(ValueError, lambda: attn.impl.set_static_kv_scales([1.0], [1.0]), "scales")
    return attn


def _common(query_lens, seq_lens, tables, slots, device):
    from vllm.v1.attention.backend import CommonAttentionMetadata

    qsl = torch.tensor(np.concatenate([[0], np.cumsum(query_lens)]), dtype=torch.int32)
    return CommonAttentionMetadata(
        query_start_loc=qsl.to(device), query_start_loc_cpu=qsl, seq_lens=torch.tensor(seq_lens, dtype=torch.int32,
                                                                                        device=device),
        num_reqs=len(query_lens), num_actual_tokens=int(sum(query_lens)), max_query_len=int(max(query_lens)),
        max_seq_len=int(max(seq_lens)), block_table_tensor=torch.from_numpy(tables).to(device),
        slot_mapping=torch.from_numpy(slots).to(device))


def _metadata_contract(va, attn, vllm_config):
    spec = attn.get_kv_cache_spec(vllm_config)
    builder = va.Hif8AttentionBackend.get_builder_cls()(spec, [attn.layer_name], vllm_config, torch.device("cpu"))
    tables = np.array([[3, 4, 0], [7, 0, 0]], dtype=np.int32)
    slots = np.array([3 * BS + 4, 4 * BS + 1, 7 * BS + 2], dtype=np.int64)
    md = builder.build(0, _common([2, 1], [21, 3], tables, slots, torch.device("cpu")))
    assert md.num_actual_tokens == 3 and md.num_reqs == 2 and md.max_seq_len == 21 and md.causal
    assert md.query_start_loc.tolist() == [0, 2, 3] and md.block_table.shape == (2, 3)
    assert builder.get_cudagraph_support(vllm_config, spec).name == "NEVER"


def main(mode: str) -> None:
    from vllm.config import CompilationConfig, DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.config.cache import CacheConfig
    from vllm.distributed import init_distributed_environment, initialize_model_parallel

    from hif8_b200 import vllm_attention as va

    gpu = mode == "gpu"
    if gpu:
        torch.cuda.set_device(0)
    _host_rules(va)
    _config_hooks(va)
    cfg = VllmConfig(device_config=DeviceConfig(device="cuda"), cache_config=CacheConfig(block_size=BS,
                                                                                         cache_dtype=DTYPE),
                     compilation_config=CompilationConfig())
    port = 29500 + os.getpid() % 200
    with set_current_vllm_config(cfg):
        init_distributed_environment(world_size=1, rank=0, distributed_init_method=f"tcp://127.0.0.1:{port}",
                                     local_rank=0, backend="gloo")
        initialize_model_parallel(1, 1)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        attn = _layer_contract(va, cfg)
        _metadata_contract(va, attn, cfg)
        if gpu:
            from _vllm_attention_gpu import forward_checks

            forward_checks(va, cfg, _layer, _common)
        torch.set_default_dtype(prev)
    print(f"vllm attention cases ({mode}): ok")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "cpu")
