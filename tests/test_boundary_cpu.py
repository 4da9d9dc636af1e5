"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every declared symbol, its host-side codec tables match the oracle, argument
contracts are enforced before any device work, and the PyTorch operators are
registered with the reference's exact schemas (no compute without a GPU)."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]

REFERENCE_SCHEMAS = {
    # reference csrc/extension/pybind.cpp:7-13
    "hif8_dynamic_quant": "vllm_ascend_hif8::hif8_dynamic_quant(Tensor x) -> (Tensor, Tensor)",
    "hif8_static_quant": "vllm_ascend_hif8::hif8_static_quant(Tensor x, Tensor fixed_scale) -> (Tensor, Tensor)",
    "hif8_scaled_decode": "vllm_ascend_hif8::hif8_scaled_decode(Tensor data, Tensor scale) -> Tensor",
    "soft_hif8_gemv": "vllm_ascend_hif8::soft_hif8_gemv(Tensor activation, Tensor weight, Tensor token_scale, "
                      "Tensor channel_scale, Tensor? bias, ScalarType output_dtype) -> Tensor",
    "soft_hif8_gemm": "vllm_ascend_hif8::soft_hif8_gemm(Tensor activation, Tensor weight, Tensor token_scale, "
                      "Tensor channel_scale, Tensor? bias, ScalarType output_dtype) -> Tensor",
    "soft_hif8_fused_gemm": "vllm_ascend_hif8::soft_hif8_fused_gemm(Tensor activation, Tensor weight, "
                            "Tensor channel_scale, Tensor? bias, ScalarType output_dtype) -> Tensor",
    "soft_hif8_static_fused_gemm": "vllm_ascend_hif8::soft_hif8_static_fused_gemm(Tensor activation, Tensor weight, "
                                   "Tensor fixed_scale, Tensor channel_scale, Tensor? bias, "
                                   "ScalarType output_dtype) -> Tensor",
}


def _declared_functions() -> list[str]:
    text = (ROOT / "include" / "hif8_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?(?:char|int|void|size_t)\s*\*?\s*(\w+)\s*\(", text, flags=re.M)


def test_cabi_exports_every_declared_symbol():
    from hif8_b200 import cabi

    names = _declared_functions()
    assert len(names) >= 14
    lib = cabi.library()
    for name in names:
        assert hasattr(lib, name), f"{name} is declared in include/hif8_b200.h but not exported"
        assert name in cabi.SIGNATURES, f"{name} has no ctypes signature"
    assert set(cabi.SIGNATURES) == set(names)


def test_model_glue_header_symbols_are_exported():
    """include/hif8_b200_model.h (the synthetic decoder's glue kernels) is
    served by the same library."""
    from hif8_b200 import cabi

    text = (ROOT / "include" / "hif8_b200_model.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*int\s+(\w+)\s*\(", text, flags=re.M)
    assert set(names) == {"hif8_model_rmsnorm", "hif8_model_silu_mul", "hif8_model_gate_mul",
                          "hif8_model_attn_prep", "hif8_model_gdn", "hif8_model_peer_allreduce_rmsnorm",
                          "hif8_model_glue_linear", "hif8_peer_alloc", "hif8_peer_open", "hif8_peer_close"}
    assert re.search(r"^\s*size_t\s+hif8_peer_buffer_bytes\s*\(", text, flags=re.M)
    import ctypes

    fn = cabi.library().hif8_peer_buffer_bytes
    fn.restype, fn.argtypes = ctypes.c_size_t, [ctypes.c_int64] * 3
    # two slots of `world` FP32 partials (max_rows x dim), one flag per (rank, CTA) for up to
    # 16 CTAs, the rank's own scratch (16 CTAs x 8 row sums + two counters), a 256-byte multiple
    want = 2 * 2 * 4 * 4096 * 4 + 2 * 16 * 4 + 16 * 8 * 4 + 16
    assert fn(2, 4, 4096) == (want + 255) // 256 * 256
    assert fn(0, 4, 4096) == 0
    lib = cabi.library()
    for name in names:
        assert hasattr(lib, name), f"{name} is declared in include/hif8_b200_model.h but not exported"


def test_model_glue_ops_are_registered():
    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    for op in ("rmsnorm", "silu_mul", "gate_mul", "glue_linear", "attn_prep", "gdn", "peer_allreduce_rmsnorm"):
        assert hasattr(torch.ops.hif8_b200, op)


def test_decoder_config_layout_and_tp_split():
    from hif8_b200.decoder import DecoderConfig

    cfg = DecoderConfig()
    full = [i for i in range(cfg.layers) if cfg.is_full(i)]
    assert full == [3, 7, 11, 15, 19, 23, 27, 31]  # every 4th layer, as Qwen3_5's layer_types
    for tp in (1, 2, 4, 8):
        assert cfg.heads % tp == 0 and cfg.lin_k_heads % tp == 0 and cfg.lin_v_heads % tp == 0
        assert cfg.intermediate % tp == 0 and cfg.vocab % tp == 0
    # per-token HiF8 projection bytes of the model (one byte per weight)
    d, v = cfg.lin_dim, cfg.lin_v_heads
    attn = (cfg.heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim) * cfg.hidden \
        + cfg.hidden * cfg.heads * cfg.head_dim
    gdn = (2 * cfg.lin_k_heads * d + 2 * v * d + 2 * v) * cfg.hidden + cfg.hidden * v * d
    mlp = 3 * cfg.intermediate * cfg.hidden
    total = len(full) * attn + (cfg.layers - len(full)) * gdn + cfg.layers * mlp
    assert 6.9e9 < total < 7.0e9


def test_cabi_codec_tables_match_oracle():
    from hif8_b200 import cabi

    lib = cabi.library()
    dec = np.zeros(256, dtype=np.uint16)
    lib.hif8_decode_table_bf16(dec.ctypes.data)
    np.testing.assert_array_equal(dec, oracle.decode_bf16_table())
    enc = np.zeros(4096, dtype=np.uint8)
    lib.hif8_encode_table(enc.ctypes.data)
    np.testing.assert_array_equal(enc, oracle.encode_lut4096())


def test_cabi_rejects_contract_violations_without_device_work():
    from hif8_b200 import cabi

    lib = cabi.library()
    fake = 256  # never dereferenced: every case fails validation first
    # soft_hif8_gemv keeps the reference's M <= 2 contract
    assert lib.soft_hif8_gemv(fake, fake, fake, fake, None, -1, 1, 3, 8, 64, fake, None) == cabi.HIF8_ERR_INVALID_ARGUMENT
    # null activation
    assert lib.soft_hif8_gemm(None, fake, fake, fake, None, -1, 1, 1, 8, 64, fake, None, 0, None) == 1
    # bad output dtype / bias dtype
    assert lib.soft_hif8_gemm(fake, fake, fake, fake, None, -1, 7, 1, 8, 64, fake, None, 0, None) == 1
    assert lib.soft_hif8_gemm(fake, fake, fake, fake, fake, 5, 1, 1, 8, 64, fake, None, 0, None) == 1
    # scale count must divide the rows
    assert lib.hif8_static_quant(fake, 1, 6, 16, fake, 4, fake, None, None) == 1
    assert lib.hif8_static_quant(fake, 3, 4, 16, fake, 1, fake, None, None) == 1
    # static fused: M <= 4
    assert lib.soft_hif8_static_fused_gemm(fake, 1, fake, fake, fake, None, -1, 1, 5, 8, 64, fake, None) == 1
    # KV: head_size must keep the FP32 sidecar aligned
    assert lib.hif8_kv_cache_write(fake, fake, 1, 1, 1, 6, 6, fake, fake, fake, fake, fake, 1, 1, None, None) == 1
    # strided pages: the block stride holds a whole block, 4-byte rows, int64 span
    dense = 16 * 2 * (64 + 4)
    for stride in (dense - 4, dense + 2, 1 << 62):
        assert lib.hif8_kv_cache_write_strided(fake, fake, 1, 1, 2, 64, 128, fake, fake, fake, fake, fake, 8, 16,
                                               stride, None, None) == 1
        assert lib.hif8_paged_attention_strided(fake, fake, fake, fake, fake, fake, 1, 1, 4, 2, 64, 8, 16, stride,
                                                1, 16, 1.0, 1, fake, None, 0, None) == 1
    assert lib.hif8_kv_cache_write_strided(fake, fake, 1, 0, 2, 64, 128, fake, fake, fake, fake, fake, 8, 16,
                                           2 * dense, None, None) == cabi.HIF8_OK  # no tokens: nothing enqueued
    # attention: heads must be a multiple of kv heads
    assert lib.hif8_paged_attention(fake, fake, fake, fake, fake, fake, 1, 1, 6, 4, 256, 8, 128, 1, 1, 1.0, 1,
                                    fake, None, 0, None) == 1
    # embedding gather: positive vocabulary and row size, pointers for any ids
    assert lib.hif8_embedding_gather(fake, fake, 0, 64, fake, 1, fake, None, None) == 1
    assert lib.hif8_embedding_gather(fake, fake, 8, 0, fake, 1, fake, None, None) == 1
    assert lib.hif8_embedding_gather(fake, fake, 8, 64, fake, -1, fake, None, None) == 1
    assert lib.hif8_embedding_gather(None, fake, 8, 64, fake, 1, fake, None, None) == 1
    assert lib.hif8_embedding_gather(fake, fake, 8, 64, None, 0, fake, None, None) == cabi.HIF8_OK  # no ids
    # dynamic quant: FP16/BF16 only, a positive scale stride, pointers for any rows
    assert lib.hif8_dynamic_quant(fake, 3, 2, 16, fake, fake, 16, None) == 1
    assert lib.hif8_dynamic_quant(fake, 1, 2, 16, fake, fake, 0, None) == 1
    assert lib.hif8_dynamic_quant(None, 1, 2, 16, fake, fake, 16, None) == 1
    assert lib.hif8_dynamic_quant(fake, 1, 2, 0, fake, fake, 16, None) == 1
    assert lib.hif8_dynamic_quant(None, 1, 0, 16, None, None, 16, None) == cabi.HIF8_OK  # no rows
    # fused dynamic linear: M <= 2 and a workspace of the reported size
    ws = lib.soft_hif8_fused_gemm_workspace_size(2, 8, 64)
    assert ws > 0 and ws % 256 == 0
    assert lib.soft_hif8_fused_gemm(fake, 1, fake, fake, None, -1, 1, 3, 8, 64, fake, fake, 1 << 20, None) == 1
    assert lib.soft_hif8_fused_gemm(fake, 1, fake, fake, None, -1, 1, 2, 8, 64, fake, fake, ws - 1, None) == 3
    assert lib.soft_hif8_fused_gemm(fake, 1, fake, fake, None, -1, 1, 2, 8, 64, fake, None, ws, None) == 3
    # the scheme's single call: the fused route needs no workspace, the other one does
    assert lib.hif8_static_linear_workspace_size(4, 8, 64, 4) == 0
    assert lib.hif8_static_linear_workspace_size(4, 8, 64, 0) == 256 + 256
    assert lib.hif8_static_linear_workspace_size(64, 4096, 4096, 4) == (
        64 * 4096 + 256 + lib.soft_hif8_gemm_workspace_size(64, 4096, 4096))
    assert lib.hif8_static_linear(fake, 3, fake, fake, fake, None, -1, 1, 2, 8, 64, 4, fake, None, 0, None) == 1
    assert lib.hif8_static_linear(fake, 1, fake, fake, fake, None, -1, 1, 5, 8, 64, 4, fake, None, 0, None) == 3
    assert lib.hif8_static_linear(fake, 1, fake, None, fake, None, -1, 1, 2, 8, 64, 4, fake, None, 0, None) == 1
    assert lib.hif8_status_string(3) == b"workspace missing or too small"


def test_paged_attention_workspace_sizes():
    from hif8_b200 import cabi

    lib = cabi.library()
    # partials of 64-key chunks: [tokens, heads, chunks, head_size + 2] FP32
    assert lib.hif8_paged_attention_workspace_size(4, 16, 256, 64) == 0  # one chunk: no partials
    assert lib.hif8_paged_attention_workspace_size(4, 16, 256, 256) == 4 * 16 * 4 * (256 + 2) * 4
    assert lib.hif8_paged_attention_workspace_size(4, 16, 256, 4096) == 4 * 16 * 64 * (256 + 2) * 4
    # a product beyond size_t is reported as SIZE_MAX, never wrapped to a small size
    size_max = (1 << 64) - 1
    assert lib.hif8_paged_attention_workspace_size(1 << 40, 1 << 10, 1024, 1 << 40) == size_max
    assert lib.hif8_paged_attention_workspace_size(0, 16, 256, 4096) == 0  # no query rows


def test_noalloc_attention_checks_arguments_before_the_scratch_size():
    """The no-alloc attention reports the same status as the workspace entry
    point for an invalid call, whatever its size; a valid call that needs
    more than the library's scratch is refused before any device work."""
    from hif8_b200 import cabi

    lib = cabi.library()
    fake = 256  # never dereferenced: every case is refused before a launch
    long_ctx = 1 << 22  # far more partials than the 8 MiB scratch holds

    def noalloc(query=fake, heads=16, kv_heads=4, ctx=long_ctx):
        return lib.hif8_paged_attention_noalloc(query, fake, fake, fake, fake, fake, 4, 4, heads, kv_heads, 256,
                                                8, 128, 1, ctx, 1.0, 1, fake, None)

    assert noalloc(query=None) == cabi.HIF8_ERR_INVALID_ARGUMENT
    assert noalloc(heads=6) == cabi.HIF8_ERR_INVALID_ARGUMENT      # heads not a multiple of kv heads
    assert noalloc(heads=68, kv_heads=4) == cabi.HIF8_ERR_INVALID_ARGUMENT  # GQA group 17 > 16
    assert noalloc() == cabi.HIF8_ERR_WORKSPACE
    assert noalloc(ctx=(1 << 62)) == cabi.HIF8_ERR_WORKSPACE       # overflowing size: SIZE_MAX


def test_torch_ops_have_reference_schemas():
    from hif8_b200 import native

    native.load_extension()
    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(torch.ops.vllm_ascend_hif8, name).default._schema) == schema


def test_ops_have_no_cpu_fallback():
    from hif8_b200 import native

    native.load_extension()
    x = torch.zeros(2, 16, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        torch.ops.vllm_ascend_hif8.hif8_static_quant(x, torch.ones(1))


def test_meta_shapes():
    from hif8_b200 import native

    native.load_extension()
    x = torch.empty(2, 3, 64, dtype=torch.bfloat16, device="meta")
    data, row_scale = torch.ops.vllm_ascend_hif8.hif8_static_quant(x, torch.empty(1, device="meta"))
    assert data.shape == x.shape and data.dtype == torch.uint8
    assert row_scale.shape == (6,) and row_scale.dtype == torch.float32
    a = torch.empty(5, 64, dtype=torch.uint8, device="meta")
    w = torch.empty(7, 64, dtype=torch.uint8, device="meta")
    out = torch.ops.vllm_ascend_hif8.soft_hif8_gemm(a, w, torch.empty(5, device="meta"), torch.empty(7, device="meta"),
                                                    None, torch.bfloat16)
    assert out.shape == (5, 7) and out.dtype == torch.bfloat16
    dec = torch.ops.vllm_ascend_hif8.hif8_scaled_decode(a, torch.empty(5, device="meta"))
    assert dec.shape == a.shape and dec.dtype == torch.bfloat16
    data, token_scale = torch.ops.vllm_ascend_hif8.hif8_dynamic_quant(x)
    assert data.shape == x.shape and data.dtype == torch.uint8 and token_scale.shape == (6,)
    lin = torch.ops.hif8_b200.static_linear(x, w, torch.empty(1, device="meta"), torch.empty(7, device="meta"))
    assert lin.shape == (2, 3, 7) and lin.dtype == torch.bfloat16
    x2 = torch.empty(2, 64, dtype=torch.float16, device="meta")
    fused = torch.ops.vllm_ascend_hif8.soft_hif8_fused_gemm(x2, w, torch.empty(7, device="meta"), None, torch.float16)
    assert fused.shape == (2, 7) and fused.dtype == torch.float16


def test_native_wrapper_contracts_raise_before_dispatch():
    from hif8_b200 import native

    with pytest.raises(TypeError):
        native.static_quant(torch.zeros(2, 4), torch.ones(1))
    with pytest.raises(TypeError):
        native.static_quant(torch.zeros(2, 4, dtype=torch.bfloat16), torch.ones(1, dtype=torch.float64))
    with pytest.raises(ValueError, match="must divide"):
        native.static_quant(torch.zeros(3, 4, dtype=torch.bfloat16), torch.ones(2))
    with pytest.raises(TypeError):
        native.soft_linear(torch.zeros(1, 4), torch.zeros(2, 4, dtype=torch.uint8), torch.ones(1), torch.ones(2),
                           output_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="incompatible K"):
        native.soft_linear(torch.zeros(1, 4, dtype=torch.uint8), torch.zeros(2, 5, dtype=torch.uint8),
                           torch.ones(1), torch.ones(2), output_dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        native.scaled_decode(torch.zeros(2, 4), torch.ones(2))
    with pytest.raises(ValueError):
        native.scaled_decode(torch.zeros(2, 2, 4, dtype=torch.uint8), torch.ones(2))
    with pytest.raises(NotImplementedError):  # the op has no CPU kernel
        native.dynamic_quant(torch.zeros(2, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="M <= 2"):
        native.soft_fused_linear(torch.zeros(3, 4, dtype=torch.bfloat16), torch.zeros(2, 4, dtype=torch.uint8),
                                 torch.ones(2), output_dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        native.soft_fused_linear(torch.zeros(1, 4), torch.zeros(2, 4, dtype=torch.uint8), torch.ones(2),
                                 output_dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        native.soft_fused_linear(torch.zeros(1, 4, dtype=torch.bfloat16), torch.zeros(2, 4, dtype=torch.uint8),
                                 torch.ones(3), output_dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        native.soft_static_fused_linear(torch.zeros(1, 4, dtype=torch.bfloat16), torch.zeros(2, 4, dtype=torch.uint8),
                                        torch.ones(2), torch.ones(2), output_dtype=torch.bfloat16)


def test_missing_extension_is_fatal(monkeypatch, tmp_path):
    from hif8_b200 import _loader, native

    monkeypatch.setattr(_loader, "_ops_loaded", False)
    monkeypatch.setattr(_loader, "_ops_error", None)
    monkeypatch.setattr(_loader, "OPS_PATH", tmp_path / "missing.so")
    native.reset_extension_cache()
    try:
        assert not native.is_available()
        with pytest.raises(native.NativeExtensionUnavailable, match="no decoded-weight or floating-point fallback"):
            native.load_extension()
    finally:
        native.reset_extension_cache()


def test_kv_layout_contract():
    from hif8_b200.kv_cache import HIF8_SCALE_BYTES, Hif8KVCacheLayout

    layout = Hif8KVCacheLayout(3, 8, 2, 16, 24)
    assert layout.key_width == 16 + HIF8_SCALE_BYTES
    assert layout.value_width == 24 + HIF8_SCALE_BYTES
    assert layout.page_size_bytes == 8 * 2 * ((16 + 4) + (24 + 4))
    assert layout.key_shape() == (3, 8, 2, 20)
    assert layout.value_shape() == (3, 8, 2, 28)
    qwen = Hif8KVCacheLayout(1, 128, 4, 256)
    assert qwen.key_width == 260 and qwen.page_size_bytes == 128 * 4 * 520
    with pytest.raises(ValueError):
        Hif8KVCacheLayout(1, 4, 1, 6)
    with pytest.raises(ValueError):
        Hif8KVCacheLayout(1, 4, 1, 8, 6)


def test_static_kv_scale_metadata(tmp_path):
    import json

    from hif8_b200.kv_cache import load_static_kv_scales

    good = tmp_path / "good"
    good.mkdir()
    (good / "hif8_metadata.json").write_text(json.dumps({
        "format": "W8A8HIF8_STATIC",
        "kv_cache": {"mode": "static_per_layer_per_head",
                     "layers": {"3": {"key_scales": [0.5, 0.75], "value_scales": [0.25, 1.0]}}}}))
    assert load_static_kv_scales(str(good)) == {3: ((0.5, 0.75), (0.25, 1.0))}
    bad = tmp_path / "bad"
    bad.mkdir()
    (bad / "hif8_metadata.json").write_text(json.dumps({
        "format": "W8A8HIF8_STATIC",
        "kv_cache": {"mode": "static_per_layer_per_head",
                     "layers": {"3": {"key_scales": [0.5, -1.0], "value_scales": [0.25, 1.0]}}}}))
    with pytest.raises(ValueError, match="invalid key_scales"):
        load_static_kv_scales(str(bad))
    missing = tmp_path / "missing"
    missing.mkdir()
    (missing / "hif8_metadata.json").write_text(json.dumps({"format": "W8A8HIF8_STATIC"}))
    with pytest.raises(ValueError, match="missing kv_cache"):
        load_static_kv_scales(str(missing))
    assert load_static_kv_scales(str(tmp_path)) is None


def test_static_scheme_parameter_contract():
    from types import SimpleNamespace

    from hif8_b200 import scheme

    def layer(scale):
        return SimpleNamespace(weight=torch.nn.Parameter(torch.zeros(4, 8, dtype=torch.uint8), requires_grad=False),
                               weight_scale=torch.nn.Parameter(torch.ones(4, 1), requires_grad=False),
                               input_scale=torch.nn.Parameter(scale, requires_grad=False))

    ok = layer(torch.tensor([0.5]))
    scheme.process_weights_after_loading(ok)
    assert ok.weight_scale.shape == (4,) and ok.input_scale.shape == (1,)
    for bad in (torch.tensor([0.0]), torch.tensor([float("inf")]), torch.tensor([-1.0]), torch.tensor([1.0, 2.0])):
        with pytest.raises(ValueError):
            scheme.process_weights_after_loading(layer(bad))
    no_scale = SimpleNamespace(weight=ok.weight, weight_scale=ok.weight_scale)
    with pytest.raises(ValueError, match="missing input_scale"):
        scheme.process_weights_after_loading(no_scale)


def test_dynamic_scheme_parameter_contract(monkeypatch):
    from types import SimpleNamespace

    from hif8_b200 import scheme

    layer = SimpleNamespace(weight=torch.nn.Parameter(torch.zeros(4, 8, dtype=torch.uint8), requires_grad=False),
                            weight_scale=torch.nn.Parameter(torch.ones(4, 1, dtype=torch.float64), requires_grad=False))
    scheme.process_dynamic_weights_after_loading(layer)
    assert layer.weight_scale.shape == (4,) and layer.weight_scale.dtype == torch.float32
    bad = SimpleNamespace(weight=torch.nn.Parameter(torch.zeros(4, 8), requires_grad=False),
                          weight_scale=layer.weight_scale)
    with pytest.raises(TypeError, match="torch.uint8"):
        scheme.process_dynamic_weights_after_loading(bad)
    short = SimpleNamespace(weight=layer.weight, weight_scale=torch.nn.Parameter(torch.ones(3), requires_grad=False))
    with pytest.raises(ValueError, match="one value per output channel"):
        scheme.process_dynamic_weights_after_loading(short)
    monkeypatch.setenv("HIF8_COMPUTE_BACKEND", "other")
    with pytest.raises(ValueError):
        scheme.process_dynamic_weights_after_loading(layer)


def test_static_scale_factor_env(monkeypatch):
    from hif8_b200 import scheme

    monkeypatch.setenv("HIF8_STATIC_SCALE_FACTOR", "2.0")
    assert scheme.static_scale_factor() == 2.0
    monkeypatch.setenv("HIF8_STATIC_SCALE_FACTOR", "-1")
    with pytest.raises(ValueError):
        scheme.static_scale_factor()
    monkeypatch.setenv("HIF8_COMPUTE_BACKEND", "other")
    with pytest.raises(ValueError):
        scheme._check_backend()
