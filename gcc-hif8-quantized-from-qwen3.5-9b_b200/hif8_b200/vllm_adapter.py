"""vLLM (CUDA) adapter: the HiF8 checkpoint's linear and embedding layers
served through vLLM's quantization-plugin interface by this build's kernels.

The reference reaches vLLM-Ascend through its scheme registry
(src/vllm_ascend_hif8/plugin.py:212-245 ``register``; the linear schemes
src/vllm_ascend_hif8/scheme.py:43-211; the embedding lookup
scheme.py:120-131).  On CUDA vLLM the same checkpoint is selected with
``quantization="hif8"``: ``Hif8Config`` reads the exporter's
``quant_model_description.json`` (weight name -> quant type) and gives every
layer its method:

* ``W8A8HIF8_STATIC`` linear -> ``Hif8StaticLinearMethod`` (uint8 weight,
  FP32 per-channel scale, one FP32 input scale; ``scheme.apply``);
* ``W8A8HIF8_SOFT`` linear -> ``Hif8SoftLinearMethod`` (dynamic per-token
  activation scale; ``scheme.apply_dynamic``);
* ``W8A8HIF8_SOFT`` token embedding -> ``Hif8EmbeddingMethod`` (the HiF8 row
  gather-decode, ``embedding_gather``);
* anything else (``FLOAT``) -> vLLM's unquantized method.

vLLM fuses q/k/v, gate/up and the gated-delta-net input projections into one
module; its components must share one quant type, and the static input scale
of a fused module is the components' shared one (the exporter stores it
under the first component, exporter.py:84-89).  The HiF8 KV cache and its
attention are the ``CUSTOM`` attention backend of ``hif8_b200.vllm_attention``,
installed by ``register()`` when ``HIF8_KV_CACHE=1``.

``register()`` is the ``vllm.general_plugins`` entry point; call it before
building an engine in the same process.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch.nn import Parameter
from vllm.model_executor.layers.linear import (
    LinearBase,
    LinearMethodBase,
    UnquantizedLinearMethod,
    register_weight_loader_v2_supported_method,
)
from vllm.model_executor.layers.quantization import QUANTIZATION_METHODS, register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig, QuantizeMethodBase
from vllm.model_executor.layers.vocab_parallel_embedding import VocabParallelEmbedding
from vllm.model_executor.parameter import ChannelQuantScaleParameter, ModelWeightParameter, PerTensorScaleParameter
from vllm.model_executor.utils import set_weight_attrs

from . import scheme
from .checkpoint import QUANT_DESCRIPTION_FILENAME

QUANT_METHOD_NAME = "hif8"
STATIC = scheme.STATIC_QUANT_TYPE
SOFT = scheme.DYNAMIC_QUANT_TYPE

# vLLM module -> checkpoint components (used when the model class does not
# provide its packed_modules_mapping)
_DEFAULT_PACKED = {
    "qkv_proj": ["q_proj", "k_proj", "v_proj"],
    "gate_up_proj": ["gate_proj", "up_proj"],
    "in_proj_qkvz": ["in_proj_qkv", "in_proj_z"],
    "in_proj_ba": ["in_proj_b", "in_proj_a"],
}
# the two spellings of the Qwen3.5 text stack (checkpoint / vLLM module tree)
_PREFIX_ALIASES = (("language_model.model.", "model.language_model."),
                   ("model.language_model.", "language_model.model."))
_UNSET = -1.0  # an input-scale slot no checkpoint tensor was loaded into


def _name_candidates(name: str) -> list[str]:
    out = [name]
    for old, new in _PREFIX_ALIASES:
        if name.startswith(old):
            out.append(new + name[len(old):])
    if name.startswith("model."):
        out.append(name[len("model."):])
    else:
        out.append("model." + name)
    return out


class Hif8Config(QuantizationConfig):
    """Quantization config of an exported HiF8 checkpoint (the contents of
    quant_model_description.json: tensor name -> quant type)."""

    def __init__(self, description: dict[str, Any]):
        super().__init__()
        self.description = {str(k): v for k, v in description.items() if isinstance(v, str)}

    def get_name(self) -> str:
        return QUANT_METHOD_NAME

    def get_supported_act_dtypes(self) -> list[torch.dtype]:
        return [torch.bfloat16, torch.float16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels

    @staticmethod
    def get_config_filenames() -> list[str]:
        return [QUANT_DESCRIPTION_FILENAME]

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "Hif8Config":
        return cls(config)

    def apply_vllm_mapper(self, hf_to_vllm_mapper) -> None:
        mapped = hf_to_vllm_mapper.apply_dict(self.description)
        self.description = {**self.description, **mapped}

    def weight_type(self, name: str) -> str | None:
        """Quant type of a checkpoint tensor, under either prefix spelling."""
        for key in _name_candidates(name):
            kind = self.description.get(key)
            if kind is not None:
                return kind
        return None

    def layer_type(self, prefix: str) -> str | None:
        """Quant type of the vLLM module at ``prefix``; a fused module's
        components must agree."""
        parent, _, leaf = prefix.rpartition(".")
        packed = self.packed_modules_mapping.get(leaf) or _DEFAULT_PACKED.get(leaf)
        if packed:
            kinds = {self.weight_type(f"{parent}.{c}.weight" if parent else f"{c}.weight") for c in packed}
            kinds.discard(None)
            if len(kinds) > 1:
                raise ValueError(f"fused module {prefix} mixes HiF8 quant types {sorted(kinds)}")
            if kinds:
                return kinds.pop()
        return self.weight_type(f"{prefix}.weight")

    def get_quant_method(self, layer: torch.nn.Module, prefix: str) -> QuantizeMethodBase | None:
        if isinstance(layer, LinearBase):
            kind = self.layer_type(prefix)
            if kind == STATIC:
                return Hif8StaticLinearMethod(self)
            if kind == SOFT:
                return Hif8SoftLinearMethod(self)
            return UnquantizedLinearMethod()
        if type(layer) is VocabParallelEmbedding and self.layer_type(prefix) == SOFT:
            return Hif8EmbeddingMethod()
        return None


def _create_hif8_linear(layer, input_size_per_partition: int, output_partition_sizes: list[int],
                        weight_loader, with_input_scale: bool) -> None:
    n = sum(output_partition_sizes)
    layer.logical_widths = output_partition_sizes
    layer.input_size_per_partition = input_size_per_partition
    layer.output_size_per_partition = n
    weight = ModelWeightParameter(data=torch.empty(n, input_size_per_partition, dtype=torch.uint8),
                                  input_dim=1, output_dim=0, weight_loader=weight_loader)
    layer.register_parameter("weight", weight)
    weight_scale = ChannelQuantScaleParameter(data=torch.empty(n, 1, dtype=torch.float32), output_dim=0,
                                              weight_loader=weight_loader)
    layer.register_parameter("weight_scale", weight_scale)
    if with_input_scale:
        input_scale = PerTensorScaleParameter(
            data=torch.full((len(output_partition_sizes),), _UNSET, dtype=torch.float32),
            weight_loader=weight_loader)
        layer.register_parameter("input_scale", input_scale)


def _replace(layer, name: str, data: torch.Tensor) -> None:
    delattr(layer, name)
    layer.register_parameter(name, Parameter(data, requires_grad=False))


def _fused_input_scale(layer) -> torch.Tensor:
    """One FP32 input scale from the slots the loader filled: a fused
    module's components share one static scale (the exporter writes it
    under the first component)."""
    values = [float(v) for v in layer.input_scale.data.reshape(-1).tolist()]
    loaded = [v for v in values if v != _UNSET]
    if not loaded:
        raise ValueError(f"{STATIC} checkpoint is missing input_scale")
    if any(v != loaded[0] for v in loaded):
        raise ValueError(f"{STATIC} fused components carry different input scales {loaded}")
    if not math.isfinite(loaded[0]) or loaded[0] <= 0.0:
        raise ValueError(f"{STATIC} input_scale must be finite and greater than zero")
    return torch.tensor([loaded[0]], dtype=torch.float32, device=layer.input_scale.device)


# vLLM's parameter-class weight loaders (v2) place every fused component's
# rows, channel scales and input-scale slot
@register_weight_loader_v2_supported_method
class Hif8StaticLinearMethod(LinearMethodBase):
    """W8A8HIF8_STATIC linear (reference scheme.py:134-211)."""

    def __init__(self, quant_config: Hif8Config):
        self.quant_config = quant_config

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        del input_size, output_size, params_dtype
        _create_hif8_linear(layer, input_size_per_partition, output_partition_sizes,
                            extra_weight_attrs.get("weight_loader"), with_input_scale=True)

    def process_weights_after_loading(self, layer) -> None:
        scale = _fused_input_scale(layer)
        _replace(layer, "weight", layer.weight.data.contiguous())
        _replace(layer, "weight_scale", layer.weight_scale.data)
        _replace(layer, "input_scale", scale)
        scheme.process_weights_after_loading(layer)

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        return scheme.apply(layer, x, bias)


@register_weight_loader_v2_supported_method
class Hif8SoftLinearMethod(LinearMethodBase):
    """W8A8HIF8_SOFT linear: dynamic per-token activation scale (reference
    scheme.py:43-116)."""

    def __init__(self, quant_config: Hif8Config):
        self.quant_config = quant_config

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        del input_size, output_size, params_dtype
        _create_hif8_linear(layer, input_size_per_partition, output_partition_sizes,
                            extra_weight_attrs.get("weight_loader"), with_input_scale=False)

    def process_weights_after_loading(self, layer) -> None:
        _replace(layer, "weight", layer.weight.data.contiguous())
        _replace(layer, "weight_scale", layer.weight_scale.data)
        scheme.process_dynamic_weights_after_loading(layer)

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        return scheme.apply_dynamic(layer, x, bias)


class Hif8EmbeddingMethod(QuantizeMethodBase):
    """HiF8 token embedding (W8A8HIF8_SOFT rows with FP32 row scales): only
    the requested rows are decoded (reference scheme.py:120-131)."""

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        del input_size, output_size
        n = sum(output_partition_sizes)
        layer.hif8_out_dtype = params_dtype
        weight = Parameter(torch.empty(n, input_size_per_partition, dtype=torch.uint8), requires_grad=False)
        set_weight_attrs(weight, {"input_dim": 1, "output_dim": 0})
        set_weight_attrs(weight, extra_weight_attrs)
        layer.register_parameter("weight", weight)
        weight_scale = Parameter(torch.zeros(n, 1, dtype=torch.float32), requires_grad=False)
        set_weight_attrs(weight_scale, {"output_dim": 0})
        set_weight_attrs(weight_scale, extra_weight_attrs)
        layer.register_parameter("weight_scale", weight_scale)

    def process_weights_after_loading(self, layer) -> None:
        from .checkpoint import Hif8Embedding

        layer.hif8_embedding = Hif8Embedding(layer.weight.data.contiguous(),
                                             layer.weight_scale.data.reshape(-1).contiguous())

    def embedding(self, layer, input_: torch.Tensor) -> torch.Tensor:
        out = layer.hif8_embedding(input_)
        return out if out.dtype == layer.hif8_out_dtype else out.to(layer.hif8_out_dtype)

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        raise NotImplementedError("the HiF8 embedding table is not used as a projection")


_registered = False


def register() -> None:
    """Make ``quantization="hif8"`` available to vLLM in this process (the
    vllm.general_plugins entry point; reference plugin.py:212-245)."""
    global _registered
    if _registered:
        return
    if QUANT_METHOD_NAME not in QUANTIZATION_METHODS:
        register_quantization_config(QUANT_METHOD_NAME)(Hif8Config)
    from .vllm_attention import install_hif8_kv_cache_adapter

    install_hif8_kv_cache_adapter()  # the HiF8 KV cache, when HIF8_KV_CACHE=1
    _registered = True
