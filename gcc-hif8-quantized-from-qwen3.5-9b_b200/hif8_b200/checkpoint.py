"""Loader for the reference exporter's HiF8 checkpoint format.

An exported W8A8HIF8_STATIC checkpoint (reference docs/checkpoint-format.md,
src/vllm_ascend_hif8/exporter.py:640-760) is a safetensors directory with

* per target projection ``<prefix>.weight`` (U8 [N, K]) and
  ``<prefix>.weight_scale`` (F32 [N, 1]); the projections are the Qwen3.5
  decoder components ``self_attn.{q,k,v,o}_proj``,
  ``mlp.{gate,up,down}_proj`` and ``linear_attn.{in_proj_qkv,in_proj_z,
  out_proj}`` (exporter.py:22-36);
* one ``<prefix>.input_scale`` (F32 [1]) per runtime linear input: the
  components that vLLM fuses into one linear share the scale written under
  the first component's name (k/v use q_proj's, up uses gate_proj's,
  in_proj_z uses in_proj_qkv's; exporter.py:75-99);
* the token embedding (``model[.language_model].embed_tokens.weight`` U8
  [vocab, hidden] + ``weight_scale``), loaded by the W8A8HIF8_SOFT method:
  gathered rows decoded with their fixed row scale, no activation quant
  (scheme.py:120-131);
* ``quant_model_description.json``: weight name -> quant type
  (exporter.py:121-138);
* ``hif8_metadata.json`` with ``kv_cache.mode == "static_per_layer_per_head"``
  and ``kv_cache.layers[<i>].{key,value}_scales`` (kv_runtime.py:206-266).

This module reads those files, validates them with the reference's rules
(fail-closed: a static checkpoint with missing or malformed scales is an
error, never a silent fallback) and builds the device objects of the hot
path: ``scheme.Hif8StaticLinear`` (fused components concatenated along N),
``Hif8Embedding`` and per-head K/V scale tensors for the KV cache.
"""

from __future__ import annotations

import json
import math
import re
from pathlib import Path

from .scheme import DYNAMIC_QUANT_TYPE, STATIC_QUANT_TYPE, Hif8StaticLinear
QUANT_DESCRIPTION_FILENAME = "quant_model_description.json"
METADATA_FILENAME = "hif8_metadata.json"
INDEX_FILENAME = "model.safetensors.index.json"
KV_MODE = "static_per_layer_per_head"

EMBEDDING_WEIGHTS = ("model.language_model.embed_tokens.weight", "model.embed_tokens.weight")

# runtime (fused) linear -> its checkpoint components, in concatenation order
# (the vLLM packing of the reference's checkpoint-format table)
FUSED_LINEARS = {
    ("self_attn", "qkv_proj"): ("q_proj", "k_proj", "v_proj"),
    ("mlp", "gate_up_proj"): ("gate_proj", "up_proj"),
    ("linear_attn", "in_proj_qkvz"): ("in_proj_qkv", "in_proj_z"),
}
# component -> the component whose input_scale it shares (exporter.py:84-89)
_CANONICAL_INPUT = {
    ("self_attn", "k_proj"): "q_proj",
    ("self_attn", "v_proj"): "q_proj",
    ("mlp", "up_proj"): "gate_proj",
    ("linear_attn", "in_proj_z"): "in_proj_qkv",
}
_LAYER_INDEX_PATTERN = re.compile(r"(?:^|\.)layers\.(\d+)(?=\.|$)")


def attention_layer_index(layer_name: str) -> int:
    """Decoder index of an attention prefix such as
    ``model.layers.31.self_attn.attn`` (kv_runtime.py:182-191)."""
    matches = _LAYER_INDEX_PATTERN.findall(str(layer_name))
    if len(matches) != 1:
        raise ValueError(f"cannot resolve one decoder layer index from HIF8 attention prefix {layer_name!r}")
    return int(matches[0])


def load_kv_scales(directory) -> dict[int, tuple[tuple[float, ...], tuple[float, ...]]] | None:
    """Static per-layer, per-head K/V scales of a checkpoint, validated
    (kv_runtime.py:206-266).  ``None`` for a legacy dynamic checkpoint (no
    metadata file, or no ``kv_cache`` entry outside a static checkpoint)."""
    metadata_path = Path(directory) / METADATA_FILENAME
    if not metadata_path.is_file():
        return None
    metadata = json.loads(metadata_path.read_text(encoding="utf-8"))
    if not isinstance(metadata, dict):
        raise ValueError(f"invalid HIF8 metadata object: {metadata_path}")
    static_checkpoint = metadata.get("format") == STATIC_QUANT_TYPE
    kv_cache = metadata.get("kv_cache")
    if kv_cache is None:
        if static_checkpoint:
            raise ValueError(f"static HIF8 checkpoint is missing kv_cache metadata: {metadata_path}")
        return None
    if not isinstance(kv_cache, dict) or kv_cache.get("mode") != KV_MODE:
        raise ValueError(f"unsupported HIF8 kv_cache metadata in {metadata_path}")
    layers = kv_cache.get("layers")
    if not isinstance(layers, dict) or not layers:
        raise ValueError(f"HIF8 kv_cache.layers is empty in {metadata_path}")
    out: dict[int, tuple[tuple[float, ...], tuple[float, ...]]] = {}
    for raw_index, entry in layers.items():
        try:
            index = int(raw_index)
        except (TypeError, ValueError) as error:
            raise ValueError(f"invalid static KV layer index {raw_index!r}") from error
        if str(index) != str(raw_index) or index < 0:
            raise ValueError(f"invalid static KV layer index {raw_index!r}")
        if not isinstance(entry, dict):
            raise ValueError(f"static KV layer {index} is not an object")
        values = []
        for kind in ("key_scales", "value_scales"):
            raw = entry.get(kind)
            if not isinstance(raw, list) or not raw:
                raise ValueError(f"static KV layer {index} has no {kind}")
            scales = tuple(float(v) for v in raw)
            if any(s <= 0.0 or not math.isfinite(s) for s in scales):
                raise ValueError(f"static KV layer {index} has invalid {kind}")
            values.append(scales)
        if len(values[0]) != len(values[1]):
            raise ValueError(f"static KV layer {index} has different K/V head counts")
        out[index] = (values[0], values[1])
    return out


def load_quant_description(directory) -> dict[str, str]:
    """``quant_model_description.json``: weight name -> quant type."""
    path = Path(directory) / QUANT_DESCRIPTION_FILENAME
    if not path.is_file():
        raise FileNotFoundError(f"HIF8 checkpoint has no {QUANT_DESCRIPTION_FILENAME}: {directory}")
    description = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(description, dict) or not all(
            isinstance(k, str) and isinstance(v, str) for k, v in description.items()):
        raise ValueError(f"invalid quant description: {path}")
    return description


def _split_prefix(prefix: str) -> tuple[str, str, str]:
    """``<layer>.<module>.<leaf>`` -> (layer prefix, module, leaf)."""
    parts = prefix.rsplit(".", 2)
    if len(parts) != 3:
        raise ValueError(f"not a decoder projection prefix: {prefix!r}")
    return parts[0], parts[1], parts[2]


def input_scale_prefix(prefix: str) -> str:
    """Checkpoint prefix whose ``input_scale`` a component consumes."""
    layer, module, leaf = _split_prefix(prefix)
    return f"{layer}.{module}.{_CANONICAL_INPUT.get((module, leaf), leaf)}"


class Hif8Embedding:
    """HiF8 token embedding: U8 rows + one FP32 scale per row; only the
    requested rows are read and decoded (reference scheme.py:120-131)."""

    def __init__(self, weight, weight_scale):
        import torch

        if weight.dtype != torch.uint8 or weight.ndim != 2:
            raise TypeError(f"{DYNAMIC_QUANT_TYPE} embedding weight must be a 2D torch.uint8 tensor, "
                            f"got {weight.dtype} {tuple(weight.shape)}")
        scale = weight_scale.to(torch.float32).reshape(-1).contiguous()
        if scale.numel() != weight.shape[0]:
            raise ValueError("embedding weight_scale must contain one value per row")
        self.weight = weight.contiguous()
        self.weight_scale = scale

    @property
    def num_embeddings(self) -> int:
        return self.weight.shape[0]

    @property
    def embedding_dim(self) -> int:
        return self.weight.shape[1]

    def __call__(self, input_ids, *, validate: bool = False):
        """BF16 ``[*input_ids.shape, hidden]``.  With ``validate=True`` the
        count of ids outside the vocabulary is read back (a host sync) and an
        ``IndexError`` raised, like the reference's ``index_select``."""
        return embedding(input_ids, self.weight, self.weight_scale, validate=validate)


def embedding(input_ids, weight, weight_scale, *, validate: bool = False):
    """Gather-decode of HiF8 embedding rows on the device (the
    ``hif8_b200::embedding_gather`` operator)."""
    import torch

    from ._loader import load_ops

    load_ops()
    ids = input_ids if input_ids.dtype == torch.int64 else input_ids.to(torch.int64)
    ids = ids.contiguous()
    if ids.storage_offset() != 0:
        ids = ids.clone()
    bad = torch.zeros(1, dtype=torch.int32, device=weight.device) if validate else None
    out = torch.ops.hif8_b200.embedding_gather(weight, weight_scale, ids, bad)
    if validate and int(bad.item()) != 0:
        raise IndexError("HIF8 embedding ids reference rows outside the vocabulary")
    return out


class Hif8Checkpoint:
    """A directory in the exported HiF8 format, read lazily with safetensors."""

    def __init__(self, directory):
        self.directory = Path(directory)
        if not self.directory.is_dir():
            raise FileNotFoundError(f"HIF8 checkpoint directory not found: {self.directory}")
        self.description = load_quant_description(self.directory)
        self._kv = load_kv_scales(self.directory)
        index = self.directory / INDEX_FILENAME
        self._files: dict[str, Path] = {}
        if index.is_file():
            weight_map = json.loads(index.read_text(encoding="utf-8")).get("weight_map", {})
            for name, shard in weight_map.items():
                self._files[name] = self.directory / shard
        else:
            from safetensors import safe_open

            for path in sorted(self.directory.glob("*.safetensors")):
                with safe_open(str(path), framework="pt") as f:
                    for name in f.keys():
                        self._files[name] = path
        if not self._files:
            raise FileNotFoundError(f"HIF8 checkpoint has no safetensors tensors: {self.directory}")

    @property
    def is_static(self) -> bool:
        return self._kv is not None or any(v == STATIC_QUANT_TYPE for v in self.description.values())

    def names(self) -> list[str]:
        return sorted(self._files)

    def has(self, name: str) -> bool:
        return name in self._files

    def tensor(self, name: str, device="cpu"):
        from safetensors import safe_open

        if name not in self._files:
            raise KeyError(f"HIF8 checkpoint has no tensor {name!r}")
        with safe_open(str(self._files[name]), framework="pt") as f:
            t = f.get_tensor(name)
        return t.to(device)

    def _quant_type(self, weight_name: str) -> str:
        if weight_name not in self.description:
            raise KeyError(f"{weight_name} is not listed in {QUANT_DESCRIPTION_FILENAME}")
        return self.description[weight_name]

    def _component(self, prefix: str, device):
        import torch

        name = f"{prefix}.weight"
        kind = self._quant_type(name)
        if kind != STATIC_QUANT_TYPE:
            raise ValueError(f"{name} is {kind}, expected {STATIC_QUANT_TYPE}")
        weight = self.tensor(name, device)
        scale = self.tensor(f"{prefix}.weight_scale", device)
        if weight.dtype != torch.uint8 or weight.ndim != 2:
            raise TypeError(f"{STATIC_QUANT_TYPE} checkpoint weight must be torch.uint8 [N, K], got "
                            f"{weight.dtype} {tuple(weight.shape)}")
        if scale.dtype != torch.float32 or scale.numel() != weight.shape[0]:
            raise ValueError(f"{prefix}.weight_scale must be float32 with one value per output channel")
        return weight, scale.reshape(-1)

    def input_scale(self, prefix: str, device="cpu"):
        return self.tensor(f"{input_scale_prefix(prefix)}.input_scale", device)

    def linear(self, prefix: str, device="cpu") -> Hif8StaticLinear:
        """One checkpoint projection, e.g. ``model.layers.0.mlp.down_proj``."""
        weight, scale = self._component(prefix, device)
        return Hif8StaticLinear(weight, scale.reshape(-1, 1), self.input_scale(prefix, device))

    def fused_linear(self, layer_prefix: str, module: str, fused: str, device="cpu") -> Hif8StaticLinear:
        """A runtime linear packed from its components along N, e.g.
        ``fused_linear("model.layers.3", "self_attn", "qkv_proj")``; every
        component must consume the same input scale."""
        import torch

        if (module, fused) not in FUSED_LINEARS:
            raise ValueError(f"unknown fused linear {module}.{fused}")
        leaves = FUSED_LINEARS[(module, fused)]
        parts = [self._component(f"{layer_prefix}.{module}.{leaf}", device) for leaf in leaves]
        k = parts[0][0].shape[1]
        if any(w.shape[1] != k for w, _ in parts):
            raise ValueError(f"{layer_prefix}.{module}.{fused}: components have different input sizes")
        scale_names = {input_scale_prefix(f"{layer_prefix}.{module}.{leaf}") for leaf in leaves}
        if len(scale_names) != 1:
            raise ValueError(f"{layer_prefix}.{module}.{fused}: components do not share one input scale")
        input_scale = self.tensor(f"{scale_names.pop()}.input_scale", device)
        weight = torch.cat([w for w, _ in parts], dim=0).contiguous()
        scale = torch.cat([s for _, s in parts], dim=0).reshape(-1, 1)
        return Hif8StaticLinear(weight, scale, input_scale)

    def embedding(self, device="cpu") -> Hif8Embedding:
        for name in EMBEDDING_WEIGHTS:
            if name in self._files:
                kind = self._quant_type(name)
                if kind != DYNAMIC_QUANT_TYPE:
                    raise ValueError(f"{name} is {kind}, expected {DYNAMIC_QUANT_TYPE}")
                prefix = name[: -len(".weight")]
                return Hif8Embedding(self.tensor(name, device), self.tensor(f"{prefix}.weight_scale", device))
        raise KeyError("HIF8 checkpoint has no token embedding")

    def kv_scales(self, layer, device="cpu"):
        """(key_scales, value_scales) F32 [kv_heads] of a full-attention
        layer, by index or attention prefix."""
        import torch

        if self._kv is None:
            raise ValueError("checkpoint has no static KV scales (legacy dynamic format)")
        index = layer if isinstance(layer, int) else attention_layer_index(layer)
        if index not in self._kv:
            raise KeyError(f"static HIF8 KV scales are missing for layer {index}")
        k, v = self._kv[index]
        return (torch.tensor(k, dtype=torch.float32, device=device),
                torch.tensor(v, dtype=torch.float32, device=device))
