"""CPU checks of the HiF8 checkpoint loader (hif8_b200.checkpoint): the
static KV metadata rules and attention-prefix parsing of the reference's
kv_runtime (tests/test_hif8_kv_runtime.py:192-250 there), and loading of an
exported-format directory written here with safetensors: single projections,
fused runtime linears with their shared input scale, the embedding and the
fail-closed errors.  No GPU."""

from __future__ import annotations

import json

import pytest
import torch
from safetensors.torch import save_file

from hif8_b200 import checkpoint


def _write_metadata(root, metadata):
    (root / checkpoint.METADATA_FILENAME).write_text(json.dumps(metadata), encoding="utf-8")


def test_static_kv_metadata_is_loaded_and_validated(tmp_path):
    metadata = {"format": "W8A8HIF8_STATIC",
                "kv_cache": {"mode": "static_per_layer_per_head",
                             "layers": {"3": {"key_scales": [0.1, 0.2], "value_scales": [0.3, 0.4]}}}}
    _write_metadata(tmp_path, metadata)
    assert checkpoint.load_kv_scales(tmp_path) == {3: ((0.1, 0.2), (0.3, 0.4))}
    metadata["kv_cache"]["layers"]["3"]["key_scales"][0] = 0.0
    _write_metadata(tmp_path, metadata)
    with pytest.raises(ValueError, match="invalid key_scales"):
        checkpoint.load_kv_scales(tmp_path)


@pytest.mark.parametrize("layers, message", [
    ({"3": {"key_scales": [0.1], "value_scales": [0.3, 0.4]}}, "different K/V head counts"),
    ({"03": {"key_scales": [0.1], "value_scales": [0.3]}}, "invalid static KV layer index"),
    ({"-1": {"key_scales": [0.1], "value_scales": [0.3]}}, "invalid static KV layer index"),
    ({"2": {"key_scales": [], "value_scales": [0.3]}}, "has no key_scales"),
    ({"2": {"key_scales": [0.1], "value_scales": [float("nan")]}}, "invalid value_scales"),
    ({"2": [0.1]}, "is not an object"),
    ({}, "kv_cache.layers is empty"),
])
def test_malformed_kv_metadata_is_rejected(tmp_path, layers, message):
    _write_metadata(tmp_path, {"format": "W8A8HIF8_STATIC",
                               "kv_cache": {"mode": "static_per_layer_per_head", "layers": layers}})
    with pytest.raises(ValueError, match=message):
        checkpoint.load_kv_scales(tmp_path)


def test_static_checkpoint_never_silently_uses_dynamic_kv(tmp_path):
    _write_metadata(tmp_path, {"format": "W8A8HIF8_STATIC"})
    with pytest.raises(ValueError, match="missing kv_cache metadata"):
        checkpoint.load_kv_scales(tmp_path)
    _write_metadata(tmp_path, {"format": "W8A8HIF8_STATIC", "kv_cache": {"mode": "dynamic", "layers": {}}})
    with pytest.raises(ValueError, match="unsupported HIF8 kv_cache metadata"):
        checkpoint.load_kv_scales(tmp_path)


def test_legacy_checkpoint_without_static_metadata_has_no_kv_scales(tmp_path):
    assert checkpoint.load_kv_scales(tmp_path) is None
    _write_metadata(tmp_path, {"format": "W8A8HIF8_SOFT"})
    assert checkpoint.load_kv_scales(tmp_path) is None


def test_attention_layer_index_accepts_real_prefixes():
    for prefix, expected in (("model.language_model.layers.3.self_attn.attn", 3),
                             ("model.layers.31.self_attn.attn", 31), ("layers.7.self_attn.attn", 7)):
        assert checkpoint.attention_layer_index(prefix) == expected
    for invalid in ("self_attn.attn", "layers.3.layers.7.attn"):
        with pytest.raises(ValueError, match="one decoder layer index"):
            checkpoint.attention_layer_index(invalid)


def test_input_scale_names_follow_the_exporter():
    p = "model.layers.5"
    assert checkpoint.input_scale_prefix(f"{p}.self_attn.k_proj") == f"{p}.self_attn.q_proj"
    assert checkpoint.input_scale_prefix(f"{p}.self_attn.v_proj") == f"{p}.self_attn.q_proj"
    assert checkpoint.input_scale_prefix(f"{p}.self_attn.o_proj") == f"{p}.self_attn.o_proj"
    assert checkpoint.input_scale_prefix(f"{p}.mlp.up_proj") == f"{p}.mlp.gate_proj"
    assert checkpoint.input_scale_prefix(f"{p}.mlp.down_proj") == f"{p}.mlp.down_proj"
    assert checkpoint.input_scale_prefix(f"{p}.linear_attn.in_proj_z") == f"{p}.linear_attn.in_proj_qkv"
    assert checkpoint.input_scale_prefix(f"{p}.linear_attn.out_proj") == f"{p}.linear_attn.out_proj"


# ------------------------------------------------ a synthetic checkpoint --

HIDDEN, VOCAB = 64, 32
COMPONENTS = {  # layer 0: full attention + MLP; layer 1: gated delta net
    "model.layers.0.self_attn.q_proj": 48, "model.layers.0.self_attn.k_proj": 16,
    "model.layers.0.self_attn.v_proj": 16, "model.layers.0.self_attn.o_proj": HIDDEN,
    "model.layers.0.mlp.gate_proj": 96, "model.layers.0.mlp.up_proj": 96,
    "model.layers.1.linear_attn.in_proj_qkv": 80, "model.layers.1.linear_attn.in_proj_z": 32,
    "model.layers.1.linear_attn.out_proj": HIDDEN,
}
INPUT_SCALES = {"model.layers.0.self_attn.q_proj": 0.011, "model.layers.0.self_attn.o_proj": 0.021,
                "model.layers.0.mlp.gate_proj": 0.031, "model.layers.1.linear_attn.in_proj_qkv": 0.041,
                "model.layers.1.linear_attn.out_proj": 0.051, "model.layers.0.mlp.down_proj": 0.061}


def make_checkpoint(root, *, shards: bool = False, seed: int = 0) -> dict[str, torch.Tensor]:
    """Write an exported-format HiF8 checkpoint (random bytes and scales)."""
    g = torch.Generator().manual_seed(seed)
    tensors: dict[str, torch.Tensor] = {}
    description: dict[str, str] = {}
    comps = dict(COMPONENTS)
    comps["model.layers.0.mlp.down_proj"] = HIDDEN
    for prefix, n in comps.items():
        k = 96 if prefix.endswith("down_proj") else HIDDEN
        # finite codes only (0x6F / 0xEF are Inf, 0x80 is NaN)
        codes = torch.randint(0, 0x6F, (n, k), generator=g, dtype=torch.int64)
        codes |= torch.randint(0, 2, (n, k), generator=g, dtype=torch.int64) << 7
        codes[codes == 0x80] = 0
        tensors[f"{prefix}.weight"] = codes.to(torch.uint8)
        tensors[f"{prefix}.weight_scale"] = (torch.rand(n, 1, generator=g) * 1e-5 + 1e-6).to(torch.float32)
        description[f"{prefix}.weight"] = "W8A8HIF8_STATIC"
    for prefix, value in INPUT_SCALES.items():
        tensors[f"{prefix}.input_scale"] = torch.tensor([value], dtype=torch.float32)
    emb = torch.randint(0, 256, (VOCAB, HIDDEN), generator=g, dtype=torch.int64).to(torch.uint8)
    tensors["model.embed_tokens.weight"] = emb
    tensors["model.embed_tokens.weight_scale"] = (torch.rand(VOCAB, 1, generator=g) * 1e-4 + 1e-6).float()
    description["model.embed_tokens.weight"] = "W8A8HIF8_SOFT"
    tensors["model.norm.weight"] = torch.ones(HIDDEN, dtype=torch.bfloat16)
    description["model.norm.weight"] = "FLOAT"
    if shards:
        names = sorted(tensors)
        half = len(names) // 2
        weight_map = {}
        for i, part in enumerate((names[:half], names[half:])):
            shard = f"model-{i + 1:05d}-of-00002.safetensors"
            save_file({n: tensors[n] for n in part}, str(root / shard))
            weight_map.update({n: shard for n in part})
        (root / checkpoint.INDEX_FILENAME).write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    else:
        save_file(tensors, str(root / "model.safetensors"))
    (root / checkpoint.QUANT_DESCRIPTION_FILENAME).write_text(json.dumps(description))
    _write_metadata(root, {"format": "W8A8HIF8_STATIC",
                           "kv_cache": {"mode": "static_per_layer_per_head",
                                        "layers": {"0": {"key_scales": [0.5, 0.25], "value_scales": [0.75, 1.5]}}}})
    return tensors


@pytest.mark.parametrize("shards", [False, True])
def test_single_projection_loads_with_its_own_scales(tmp_path, shards):
    tensors = make_checkpoint(tmp_path, shards=shards)
    ckpt = checkpoint.Hif8Checkpoint(tmp_path)
    assert ckpt.is_static
    layer = ckpt.linear("model.layers.0.mlp.down_proj")
    assert torch.equal(layer.weight, tensors["model.layers.0.mlp.down_proj.weight"])
    assert torch.equal(layer.weight_scale, tensors["model.layers.0.mlp.down_proj.weight_scale"].reshape(-1))
    assert layer.weight_scale.shape == (HIDDEN,)
    assert float(layer.input_scale) == pytest.approx(0.061)
    assert (layer.out_features, layer.in_features) == (HIDDEN, 96)


@pytest.mark.parametrize("module, fused, leaves, scale", [
    ("self_attn", "qkv_proj", ("q_proj", "k_proj", "v_proj"), 0.011),
    ("mlp", "gate_up_proj", ("gate_proj", "up_proj"), 0.031),
    ("linear_attn", "in_proj_qkvz", ("in_proj_qkv", "in_proj_z"), 0.041),
])
def test_fused_linear_concatenates_components_and_shares_the_input_scale(tmp_path, module, fused, leaves, scale):
    tensors = make_checkpoint(tmp_path)
    layer_prefix = "model.layers.1" if module == "linear_attn" else "model.layers.0"
    layer = checkpoint.Hif8Checkpoint(tmp_path).fused_linear(layer_prefix, module, fused)
    parts = [f"{layer_prefix}.{module}.{leaf}" for leaf in leaves]
    assert torch.equal(layer.weight, torch.cat([tensors[f"{p}.weight"] for p in parts]))
    assert torch.equal(layer.weight_scale, torch.cat([tensors[f"{p}.weight_scale"].reshape(-1) for p in parts]))
    assert float(layer.input_scale) == pytest.approx(scale)
    # a component alone reads the shared (canonical) input scale too
    assert float(checkpoint.Hif8Checkpoint(tmp_path).linear(parts[-1]).input_scale) == pytest.approx(scale)


def test_embedding_and_kv_scales(tmp_path):
    tensors = make_checkpoint(tmp_path)
    ckpt = checkpoint.Hif8Checkpoint(tmp_path)
    emb = ckpt.embedding()
    assert torch.equal(emb.weight, tensors["model.embed_tokens.weight"])
    assert emb.weight_scale.shape == (VOCAB,)
    assert (emb.num_embeddings, emb.embedding_dim) == (VOCAB, HIDDEN)
    k, v = ckpt.kv_scales(0)
    assert k.tolist() == [0.5, 0.25] and v.tolist() == [0.75, 1.5]
    k2, _ = ckpt.kv_scales("model.layers.0.self_attn.attn")
    assert torch.equal(k, k2)
    with pytest.raises(KeyError, match="missing for layer 4"):
        ckpt.kv_scales(4)


def test_loader_fails_closed(tmp_path):
    tensors = make_checkpoint(tmp_path)
    ckpt = checkpoint.Hif8Checkpoint(tmp_path)
    with pytest.raises(ValueError, match="expected W8A8HIF8_STATIC"):
        ckpt._component("model.embed_tokens", "cpu")
    with pytest.raises(KeyError, match="not listed"):
        ckpt.linear("model.layers.7.mlp.down_proj")
    with pytest.raises(ValueError, match="unknown fused linear"):
        ckpt.fused_linear("model.layers.0", "mlp", "qkv_proj")
    # a non-positive or non-scalar input scale is refused by the scheme's checks
    bad = dict(tensors)
    bad["model.layers.0.mlp.down_proj.input_scale"] = torch.tensor([0.0])
    save_file(bad, str(tmp_path / "model.safetensors"))
    with pytest.raises(ValueError, match="finite and greater than zero"):
        checkpoint.Hif8Checkpoint(tmp_path).linear("model.layers.0.mlp.down_proj")
    bad["model.layers.0.mlp.down_proj.input_scale"] = torch.tensor([0.1, 0.2])
    save_file(bad, str(tmp_path / "model.safetensors"))
    with pytest.raises(ValueError, match="one input_scale value"):
        checkpoint.Hif8Checkpoint(tmp_path).linear("model.layers.0.mlp.down_proj")
    # weights must stay HiF8 bytes
    bad["model.layers.0.mlp.down_proj.input_scale"] = torch.tensor([0.1])
    bad["model.layers.0.mlp.down_proj.weight"] = bad["model.layers.0.mlp.down_proj.weight"].to(torch.int16)
    save_file(bad, str(tmp_path / "model.safetensors"))
    with pytest.raises(TypeError, match="must be torch.uint8"):
        checkpoint.Hif8Checkpoint(tmp_path).linear("model.layers.0.mlp.down_proj")
    # a static checkpoint without KV metadata is an error at open
    _write_metadata(tmp_path, {"format": "W8A8HIF8_STATIC"})
    with pytest.raises(ValueError, match="missing kv_cache metadata"):
        checkpoint.Hif8Checkpoint(tmp_path)
    (tmp_path / checkpoint.QUANT_DESCRIPTION_FILENAME).unlink()
    with pytest.raises(FileNotFoundError, match="quant_model_description"):
        checkpoint.Hif8Checkpoint(tmp_path)
