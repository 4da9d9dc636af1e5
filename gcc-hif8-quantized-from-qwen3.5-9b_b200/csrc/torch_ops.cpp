// PyTorch operator registrations over the hif8_b200 C ABI.
//
// Namespace vllm_ascend_hif8 carries the reference plugin's operators with
// their exact schemas (reference csrc/extension/pybind.cpp:6-14), a CUDA
// implementation and Meta (shape) implementations, so `native.py`-style
// callers that look up torch.ops.vllm_ascend_hif8.<op> reach these kernels
// unchanged.  The argument checks and their messages follow the reference
// bridge (csrc/extension/hif8_native.cpp:131-316), with "NPU" read as "CUDA".
// Namespace hif8_b200 carries the fused KV operators that have no single
// reference operator (they replace Python sequences in kv_runtime.py).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdint>
#include <limits>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/hif8_b200.h"
#include "../../include/hif8_b200_model.h"

namespace {

void CheckStatus(int status, const char *operation) {
  TORCH_CHECK(status == HIF8_OK, operation, " failed: ", hif8_status_string(status),
              status == HIF8_ERR_CUDA ? std::string(" (") + hif8_last_error() + ")" : std::string());
}

void CheckCudaTensor(const at::Tensor &tensor, const char *name) {
  TORCH_CHECK(tensor.defined(), name, " must be defined");
  TORCH_CHECK(tensor.is_cuda(), name, " must be a CUDA tensor, got ", tensor.device());
  TORCH_CHECK(tensor.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(tensor.storage_offset() == 0, name, " must have storage_offset == 0");
}

void CheckSameDevice(const at::Tensor &tensor, const at::Device &device, const char *name) {
  TORCH_CHECK(tensor.device() == device, name, " must be on ", device, ", got ", tensor.device());
}

void CheckPositiveDimensions(const at::Tensor &tensor, const char *name) {
  for (int64_t dim = 0; dim < tensor.dim(); ++dim)
    TORCH_CHECK(tensor.size(dim) > 0, name, " dimensions must be positive, got ", tensor.sizes());
}

void CheckFitsUint32(int64_t value, const char *name) {
  TORCH_CHECK(value > 0 && static_cast<uint64_t>(value) <= std::numeric_limits<uint32_t>::max(), name,
              " must fit a positive uint32, got ", value);
}

int DtypeCode(at::ScalarType t) {
  return t == at::ScalarType::BFloat16 ? HIF8_DTYPE_BF16 : HIF8_DTYPE_F16;
}

void *Stream(const at::Tensor &t) {
  return static_cast<void *>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void ValidateSoftLinear(const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &token_scale,
                        const at::Tensor &channel_scale, const std::optional<at::Tensor> &bias,
                        at::ScalarType output_type, bool gemv) {
  CheckCudaTensor(activation, "activation");
  CheckCudaTensor(weight, "weight");
  CheckCudaTensor(token_scale, "token_scale");
  CheckCudaTensor(channel_scale, "channel_scale");
  TORCH_CHECK(activation.scalar_type() == at::ScalarType::Byte, "activation must have dtype torch.uint8");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte, "weight must have dtype torch.uint8");
  TORCH_CHECK(token_scale.scalar_type() == at::ScalarType::Float, "token_scale must have dtype torch.float32");
  TORCH_CHECK(channel_scale.scalar_type() == at::ScalarType::Float, "channel_scale must have dtype torch.float32");
  TORCH_CHECK(activation.dim() == 2, "activation must have shape [M, K]");
  TORCH_CHECK(weight.dim() == 2, "weight must have shape [N, K]");
  TORCH_CHECK(token_scale.dim() == 1, "token_scale must have shape [M]");
  TORCH_CHECK(channel_scale.dim() == 1, "channel_scale must have shape [N]");
  CheckPositiveDimensions(activation, "activation");
  CheckPositiveDimensions(weight, "weight");
  const int64_t m = activation.size(0), k = activation.size(1), n = weight.size(0);
  TORCH_CHECK(weight.size(1) == k, "activation and weight K dimensions differ: ", k, " != ", weight.size(1));
  TORCH_CHECK(token_scale.numel() == m, "token_scale must contain one value per activation row");
  TORCH_CHECK(channel_scale.numel() == n, "channel_scale must contain one value per output channel");
  TORCH_CHECK(gemv ? m <= 2 : m > 0, gemv ? "soft_hif8_gemv requires M <= 2" : "soft_hif8_gemm requires M > 0");
  CheckFitsUint32(m, "M");
  CheckFitsUint32(n, "N");
  CheckFitsUint32(k, "K");
  const auto device = activation.device();
  CheckSameDevice(weight, device, "weight");
  CheckSameDevice(token_scale, device, "token_scale");
  CheckSameDevice(channel_scale, device, "channel_scale");
  if (bias.has_value()) {
    CheckCudaTensor(*bias, "bias");
    CheckSameDevice(*bias, device, "bias");
    TORCH_CHECK(bias->dim() == 1, "bias must have shape [N]");
    TORCH_CHECK(bias->numel() == n, "bias must contain N values");
    TORCH_CHECK(bias->scalar_type() == at::ScalarType::Half || bias->scalar_type() == at::ScalarType::BFloat16,
                "bias must have dtype torch.float16 or torch.bfloat16");
  }
  TORCH_CHECK(output_type == at::ScalarType::Half || output_type == at::ScalarType::BFloat16,
              "output_dtype must be torch.float16 or torch.bfloat16");
}

std::tuple<at::Tensor, at::Tensor> Hif8StaticQuant(const at::Tensor &x, const at::Tensor &fixed_scale) {
  CheckCudaTensor(x, "x");
  CheckCudaTensor(fixed_scale, "fixed_scale");
  TORCH_CHECK(x.scalar_type() == at::ScalarType::Half || x.scalar_type() == at::ScalarType::BFloat16,
              "x must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(fixed_scale.scalar_type() == at::ScalarType::Float, "fixed_scale must have dtype torch.float32");
  TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
  TORCH_CHECK(fixed_scale.dim() == 1, "fixed_scale must have shape [scale_count]");
  CheckPositiveDimensions(x, "x");
  CheckPositiveDimensions(fixed_scale, "fixed_scale");
  const int64_t rows = x.numel() / x.size(-1);
  TORCH_CHECK(rows % fixed_scale.numel() == 0, "fixed_scale count must divide the activation row count");
  CheckFitsUint32(rows, "activation row count");
  CheckFitsUint32(x.size(-1), "K");
  CheckFitsUint32(fixed_scale.numel(), "fixed scale count");
  CheckSameDevice(fixed_scale, x.device(), "fixed_scale");
  c10::cuda::CUDAGuard guard(x.device());
  auto data = at::empty(x.sizes(), x.options().dtype(at::kByte));
  auto row_scale = at::empty({rows}, x.options().dtype(at::kFloat));
  CheckStatus(hif8_static_quant(x.data_ptr(), DtypeCode(x.scalar_type()), rows, x.size(-1),
                                fixed_scale.data_ptr<float>(), fixed_scale.numel(), data.data_ptr<uint8_t>(),
                                row_scale.data_ptr<float>(), Stream(x)),
              "hif8_static_quant");
  return {data, row_scale};
}

at::Tensor Hif8ScaledDecode(const at::Tensor &data, const at::Tensor &scale) {
  CheckCudaTensor(data, "data");
  CheckCudaTensor(scale, "scale");
  TORCH_CHECK(data.scalar_type() == at::ScalarType::Byte, "data must have dtype torch.uint8");
  TORCH_CHECK(scale.scalar_type() == at::ScalarType::Float, "scale must have dtype torch.float32");
  TORCH_CHECK(data.dim() == 2, "data must have shape [rows, K]");
  TORCH_CHECK(scale.dim() == 1, "scale must have shape [rows]");
  CheckPositiveDimensions(data, "data");
  TORCH_CHECK(scale.numel() == data.size(0), "scale must contain one value per data row");
  CheckFitsUint32(data.size(0), "row count");
  CheckFitsUint32(data.size(1), "K");
  CheckSameDevice(scale, data.device(), "scale");
  c10::cuda::CUDAGuard guard(data.device());
  auto out = at::empty(data.sizes(), data.options().dtype(at::kBFloat16));
  CheckStatus(hif8_scaled_decode(data.data_ptr<uint8_t>(), data.size(0), data.size(1), data.size(1),
                                 scale.data_ptr<float>(), reinterpret_cast<uint16_t *>(out.data_ptr()), Stream(data)),
              "hif8_scaled_decode");
  return out;
}

at::Tensor SoftHif8Linear(const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &token_scale,
                          const at::Tensor &channel_scale, const std::optional<at::Tensor> &bias,
                          at::ScalarType output_type, bool gemv) {
  ValidateSoftLinear(activation, weight, token_scale, channel_scale, bias, output_type, gemv);
  c10::cuda::CUDAGuard guard(activation.device());
  const int64_t m = activation.size(0), k = activation.size(1), n = weight.size(0);
  auto out = at::empty({m, n}, activation.options().dtype(output_type));
  const void *bias_ptr = bias.has_value() ? bias->data_ptr() : nullptr;
  const int bias_dtype = bias.has_value() ? DtypeCode(bias->scalar_type()) : HIF8_DTYPE_NONE;
  if (gemv) {
    CheckStatus(soft_hif8_gemv(activation.data_ptr<uint8_t>(), weight.data_ptr<uint8_t>(),
                               token_scale.data_ptr<float>(), channel_scale.data_ptr<float>(), bias_ptr, bias_dtype,
                               DtypeCode(output_type), m, n, k, out.data_ptr(), Stream(activation)),
                "soft_hif8_gemv");
  } else {
    const size_t ws_bytes = soft_hif8_gemm_workspace_size(m, n, k);
    at::Tensor ws;
    if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, activation.options().dtype(at::kByte));
    CheckStatus(soft_hif8_gemm(activation.data_ptr<uint8_t>(), weight.data_ptr<uint8_t>(),
                               token_scale.data_ptr<float>(), channel_scale.data_ptr<float>(), bias_ptr, bias_dtype,
                               DtypeCode(output_type), m, n, k, out.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr,
                               ws_bytes, Stream(activation)),
                "soft_hif8_gemm");
  }
  return out;
}

at::Tensor SoftHif8Gemv(const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &token_scale,
                        const at::Tensor &channel_scale, const std::optional<at::Tensor> &bias,
                        at::ScalarType output_type) {
  return SoftHif8Linear(activation, weight, token_scale, channel_scale, bias, output_type, true);
}

at::Tensor SoftHif8Gemm(const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &token_scale,
                        const at::Tensor &channel_scale, const std::optional<at::Tensor> &bias,
                        at::ScalarType output_type) {
  return SoftHif8Linear(activation, weight, token_scale, channel_scale, bias, output_type, false);
}

at::Tensor SoftHif8StaticFusedGemm(const at::Tensor &activation, const at::Tensor &weight,
                                   const at::Tensor &fixed_scale, const at::Tensor &channel_scale,
                                   const std::optional<at::Tensor> &bias, at::ScalarType output_type) {
  CheckCudaTensor(activation, "activation");
  CheckCudaTensor(weight, "weight");
  CheckCudaTensor(fixed_scale, "fixed_scale");
  CheckCudaTensor(channel_scale, "channel_scale");
  TORCH_CHECK(activation.scalar_type() == at::ScalarType::Half || activation.scalar_type() == at::ScalarType::BFloat16,
              "activation must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte, "weight must have dtype torch.uint8");
  TORCH_CHECK(fixed_scale.scalar_type() == at::ScalarType::Float, "fixed_scale must have dtype torch.float32");
  TORCH_CHECK(channel_scale.scalar_type() == at::ScalarType::Float, "channel_scale must have dtype torch.float32");
  TORCH_CHECK(activation.dim() == 2, "activation must have shape [M, K]");
  TORCH_CHECK(weight.dim() == 2, "weight must have shape [N, K]");
  TORCH_CHECK(fixed_scale.dim() == 1 && fixed_scale.numel() == 1, "fixed_scale must have shape [1]");
  TORCH_CHECK(channel_scale.dim() == 1, "channel_scale must have shape [N]");
  CheckPositiveDimensions(activation, "activation");
  CheckPositiveDimensions(weight, "weight");
  TORCH_CHECK(activation.size(0) <= 4, "soft_hif8_static_fused_gemm requires M <= 4");
  TORCH_CHECK(activation.size(1) == weight.size(1), "activation and weight K dimensions differ: ", activation.size(1),
              " != ", weight.size(1));
  TORCH_CHECK(channel_scale.numel() == weight.size(0), "channel_scale must contain one value per output channel");
  CheckFitsUint32(activation.size(0), "M");
  CheckFitsUint32(weight.size(0), "N");
  CheckFitsUint32(activation.size(1), "K");
  CheckSameDevice(weight, activation.device(), "weight");
  CheckSameDevice(fixed_scale, activation.device(), "fixed_scale");
  CheckSameDevice(channel_scale, activation.device(), "channel_scale");
  if (bias.has_value()) {
    CheckCudaTensor(*bias, "bias");
    CheckSameDevice(*bias, activation.device(), "bias");
    TORCH_CHECK(bias->dim() == 1, "bias must have shape [N]");
    TORCH_CHECK(bias->numel() == weight.size(0), "bias must contain N values");
    TORCH_CHECK(bias->scalar_type() == at::ScalarType::Half || bias->scalar_type() == at::ScalarType::BFloat16,
                "bias must have dtype torch.float16 or torch.bfloat16");
  }
  TORCH_CHECK(output_type == at::ScalarType::Half || output_type == at::ScalarType::BFloat16,
              "output_dtype must be torch.float16 or torch.bfloat16");
  c10::cuda::CUDAGuard guard(activation.device());
  const int64_t m = activation.size(0), k = activation.size(1), n = weight.size(0);
  auto out = at::empty({m, n}, activation.options().dtype(output_type));
  CheckStatus(soft_hif8_static_fused_gemm(activation.data_ptr(), DtypeCode(activation.scalar_type()),
                                          weight.data_ptr<uint8_t>(), fixed_scale.data_ptr<float>(),
                                          channel_scale.data_ptr<float>(), bias.has_value() ? bias->data_ptr() : nullptr,
                                          bias.has_value() ? DtypeCode(bias->scalar_type()) : HIF8_DTYPE_NONE,
                                          DtypeCode(output_type), m, n, k, out.data_ptr(), Stream(activation)),
              "soft_hif8_static_fused_gemm");
  return out;
}

// Dynamic per-row quant (reference hif8_native.cpp:433-486): data like x
// (uint8), token scales as a [rows] view of stride 16 (the reference's
// layout), checks and messages of the reference wrapper.
std::tuple<at::Tensor, at::Tensor> Hif8DynamicQuant(const at::Tensor &x) {
  CheckCudaTensor(x, "x");
  TORCH_CHECK(x.scalar_type() == at::ScalarType::Half || x.scalar_type() == at::ScalarType::BFloat16,
              "x must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
  CheckPositiveDimensions(x, "x");
  const int64_t rows = x.numel() / x.size(-1);
  CheckFitsUint32(rows, "activation row count");
  CheckFitsUint32(x.size(-1), "K");
  c10::cuda::CUDAGuard guard(x.device());
  auto data = at::empty(x.sizes(), x.options().dtype(at::kByte));
  constexpr int64_t kScaleStride = 16;
  auto storage = at::empty({rows * kScaleStride}, x.options().dtype(at::kFloat));
  auto token_scale = storage.as_strided({rows}, {kScaleStride});
  CheckStatus(hif8_dynamic_quant(x.data_ptr(), DtypeCode(x.scalar_type()), rows, x.size(-1),
                                 data.data_ptr<uint8_t>(), storage.data_ptr<float>(), kScaleStride, Stream(x)),
              "hif8_dynamic_quant");
  return {data, token_scale};
}

// Dynamic quant + linear (reference hif8_native.cpp:676-760), M <= 2.
at::Tensor SoftHif8FusedGemm(const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &channel_scale,
                             const std::optional<at::Tensor> &bias, at::ScalarType output_type) {
  CheckCudaTensor(activation, "activation");
  CheckCudaTensor(weight, "weight");
  CheckCudaTensor(channel_scale, "channel_scale");
  TORCH_CHECK(activation.scalar_type() == at::ScalarType::Half || activation.scalar_type() == at::ScalarType::BFloat16,
              "activation must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte, "weight must have dtype torch.uint8");
  TORCH_CHECK(channel_scale.scalar_type() == at::ScalarType::Float, "channel_scale must have dtype torch.float32");
  TORCH_CHECK(activation.dim() == 2, "activation must have shape [M, K]");
  TORCH_CHECK(weight.dim() == 2, "weight must have shape [N, K]");
  TORCH_CHECK(channel_scale.dim() == 1, "channel_scale must have shape [N]");
  CheckPositiveDimensions(activation, "activation");
  CheckPositiveDimensions(weight, "weight");
  TORCH_CHECK(activation.size(0) <= 2, "soft_hif8_fused_gemm requires M <= 2");
  TORCH_CHECK(activation.size(1) == weight.size(1), "activation and weight K dimensions differ: ", activation.size(1),
              " != ", weight.size(1));
  TORCH_CHECK(channel_scale.numel() == weight.size(0), "channel_scale must contain one value per output channel");
  CheckFitsUint32(activation.size(0), "M");
  CheckFitsUint32(weight.size(0), "N");
  CheckFitsUint32(activation.size(1), "K");
  CheckSameDevice(weight, activation.device(), "weight");
  CheckSameDevice(channel_scale, activation.device(), "channel_scale");
  int bias_dtype = HIF8_DTYPE_NONE;
  if (bias.has_value()) {
    CheckCudaTensor(*bias, "bias");
    CheckSameDevice(*bias, activation.device(), "bias");
    TORCH_CHECK(bias->dim() == 1, "bias must have shape [N]");
    TORCH_CHECK(bias->numel() == weight.size(0), "bias must contain N values");
    TORCH_CHECK(bias->scalar_type() == at::ScalarType::Half || bias->scalar_type() == at::ScalarType::BFloat16,
                "bias must have dtype torch.float16 or torch.bfloat16");
    bias_dtype = DtypeCode(bias->scalar_type());
  }
  TORCH_CHECK(output_type == at::ScalarType::Half || output_type == at::ScalarType::BFloat16,
              "output_dtype must be torch.float16 or torch.bfloat16");
  c10::cuda::CUDAGuard guard(activation.device());
  const int64_t m = activation.size(0), k = activation.size(1), n = weight.size(0);
  auto out = at::empty({m, n}, activation.options().dtype(output_type));
  const size_t ws_bytes = soft_hif8_fused_gemm_workspace_size(m, n, k);
  auto ws = at::empty({(int64_t)ws_bytes}, activation.options().dtype(at::kByte));
  CheckStatus(soft_hif8_fused_gemm(activation.data_ptr(), DtypeCode(activation.scalar_type()),
                                   weight.data_ptr<uint8_t>(), channel_scale.data_ptr<float>(),
                                   bias.has_value() ? bias->data_ptr() : nullptr, bias_dtype,
                                   DtypeCode(output_type), m, n, k, out.data_ptr(), ws.data_ptr(), ws_bytes,
                                   Stream(activation)),
              "soft_hif8_fused_gemm");
  return out;
}

// HiF8 token embedding (reference scheme.py:120-131): gather + decode of the
// requested rows only; [*ids.shape, hidden] BF16.
at::Tensor Hif8EmbeddingGather(const at::Tensor &weight, const at::Tensor &weight_scale, const at::Tensor &ids,
                               const std::optional<at::Tensor> &bad_ids) {
  CheckCudaTensor(weight, "weight");
  CheckCudaTensor(weight_scale, "weight_scale");
  CheckCudaTensor(ids, "ids");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte && weight.dim() == 2,
              "weight must be a uint8 [vocab, hidden] tensor");
  TORCH_CHECK(weight_scale.scalar_type() == at::ScalarType::Float && weight_scale.numel() == weight.size(0),
              "weight_scale must be float32 with one value per embedding row");
  TORCH_CHECK(ids.scalar_type() == at::kLong, "ids must have dtype torch.int64");
  CheckSameDevice(weight_scale, weight.device(), "weight_scale");
  CheckSameDevice(ids, weight.device(), "ids");
  int32_t *bad = nullptr;
  if (bad_ids.has_value()) {
    CheckCudaTensor(*bad_ids, "bad_ids");
    TORCH_CHECK(bad_ids->scalar_type() == at::kInt && bad_ids->numel() >= 1, "bad_ids must be int32");
    bad = bad_ids->data_ptr<int32_t>();
  }
  std::vector<int64_t> shape(ids.sizes().begin(), ids.sizes().end());
  shape.push_back(weight.size(1));
  c10::cuda::CUDAGuard guard(weight.device());
  at::Tensor out = at::empty(shape, weight.options().dtype(at::kBFloat16));
  CheckStatus(hif8_embedding_gather(weight.data_ptr<uint8_t>(), weight_scale.data_ptr<float>(), weight.size(0),
                                    weight.size(1), ids.data_ptr<int64_t>(), ids.numel(),
                                    reinterpret_cast<uint16_t *>(out.data_ptr()), bad, Stream(weight)),
              "hif8_embedding_gather");
  return out;
}

// --------------------------------------------------------------- KV ops --

// A cache plane: uint8 [num_blocks, block_size, heads, head_size + 4] with
// dense rows and row groups, whose blocks may sit further apart (one plane
// of vLLM's block-major page [num_blocks, 2, block_size, heads, width]).
// Returns the block stride in bytes.
int64_t CacheBlockStride(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.defined() && t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kByte && t.dim() == 4,
              name, " must be uint8 [num_blocks, block_size, heads, head_size + 4]");
  auto dense_dim = [&](int dim, int64_t want) { return t.size(dim) == 1 || t.stride(dim) == want; };
  const int64_t group = t.size(2) * t.size(3), block = t.size(1) * group;
  TORCH_CHECK(dense_dim(3, 1) && dense_dim(2, t.size(3)) && dense_dim(1, group),
              name, " must have dense rows and row groups");
  const int64_t stride = t.size(0) == 1 ? block : t.stride(0);
  TORCH_CHECK(stride >= block, name, " blocks must not overlap");
  return stride;
}

void Hif8KvCacheWrite(const at::Tensor &key, const at::Tensor &value, const at::Tensor &key_scale,
                      const at::Tensor &value_scale, const at::Tensor &slot_mapping, at::Tensor key_cache,
                      at::Tensor value_cache, const std::optional<at::Tensor> &bad_slots) {
  TORCH_CHECK(key.is_cuda() && value.is_cuda(), "key/value must be CUDA tensors");
  TORCH_CHECK(key.dim() == 3 && value.sizes() == key.sizes(), "key/value must have shape [tokens, heads, head_size]");
  TORCH_CHECK(key.scalar_type() == value.scalar_type() &&
                  (key.scalar_type() == at::kBFloat16 || key.scalar_type() == at::kHalf),
              "key/value must be float16 or bfloat16");
  TORCH_CHECK(key.stride(2) == 1 && key.stride(1) == key.size(2) && value.stride(2) == 1 &&
                  value.stride(1) == value.size(2) && key.stride(0) == value.stride(0),
              "key/value rows must be contiguous [heads, head_size] blocks with a shared token stride");
  CheckCudaTensor(key_scale, "key_scale");
  CheckCudaTensor(value_scale, "value_scale");
  CheckCudaTensor(slot_mapping, "slot_mapping");
  const int64_t block_stride = CacheBlockStride(key_cache, "key_cache");
  TORCH_CHECK(CacheBlockStride(value_cache, "value_cache") == block_stride,
              "key_cache and value_cache must have the same block stride");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kLong && slot_mapping.dim() == 1 &&
                  slot_mapping.numel() >= key.size(0),
              "slot_mapping must be int64 with one slot per token");
  TORCH_CHECK(key_scale.scalar_type() == at::kFloat && key_scale.numel() == key.size(1) &&
                  value_scale.scalar_type() == at::kFloat && value_scale.numel() == key.size(1),
              "key_scale/value_scale must be float32 with one value per KV head");
  TORCH_CHECK(key_cache.scalar_type() == at::kByte && key_cache.dim() == 4 && key_cache.size(2) == key.size(1) &&
                  key_cache.size(3) == key.size(2) + 4 && value_cache.sizes() == key_cache.sizes() &&
                  value_cache.scalar_type() == at::kByte,
              "caches must be uint8 [num_blocks, block_size, heads, head_size + 4]");
  int32_t *bad = nullptr;
  if (bad_slots.has_value()) {
    CheckCudaTensor(*bad_slots, "bad_slots");
    TORCH_CHECK(bad_slots->scalar_type() == at::kInt && bad_slots->numel() >= 1, "bad_slots must be int32");
    bad = bad_slots->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard guard(key.device());
  CheckStatus(hif8_kv_cache_write_strided(key.data_ptr(), value.data_ptr(), DtypeCode(key.scalar_type()),
                                          key.size(0), key.size(1), key.size(2), key.stride(0),
                                          key_scale.data_ptr<float>(), value_scale.data_ptr<float>(),
                                          slot_mapping.data_ptr<int64_t>(), key_cache.data_ptr<uint8_t>(),
                                          value_cache.data_ptr<uint8_t>(), key_cache.size(0), key_cache.size(1),
                                          block_stride, bad, Stream(key)),
              "hif8_kv_cache_write");
}

at::Tensor Hif8PagedAttention(const at::Tensor &query, const at::Tensor &key_cache, const at::Tensor &value_cache,
                              const at::Tensor &block_tables, const at::Tensor &seq_lens,
                              const at::Tensor &query_start, int64_t max_seq_len, double softmax_scale,
                              bool causal) {
  CheckCudaTensor(query, "query");
  const int64_t block_stride = CacheBlockStride(key_cache, "key_cache");
  TORCH_CHECK(CacheBlockStride(value_cache, "value_cache") == block_stride,
              "key_cache and value_cache must have the same block stride");
  CheckCudaTensor(block_tables, "block_tables");
  CheckCudaTensor(seq_lens, "seq_lens");
  CheckCudaTensor(query_start, "query_start");
  TORCH_CHECK(query.scalar_type() == at::kBFloat16 && query.dim() == 3, "query must be bfloat16 [tokens, heads, D]");
  TORCH_CHECK(key_cache.scalar_type() == at::kByte && key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes(),
              "caches must be uint8 [num_blocks, block_size, kv_heads, D + 4]");
  TORCH_CHECK(key_cache.size(3) == query.size(2) + 4, "cache row width must be head_size + 4");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2, "block_tables must be int32 [B, max_blocks]");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.numel() == block_tables.size(0), "seq_lens must be int32 [B]");
  TORCH_CHECK(query_start.scalar_type() == at::kInt && query_start.numel() == block_tables.size(0) + 1,
              "query_start must be int32 [B + 1]");
  c10::cuda::CUDAGuard guard(query.device());
  auto out = at::empty_like(query);
  const int64_t tokens = query.size(0), heads = query.size(1), d = query.size(2);
  const size_t ws_bytes = hif8_paged_attention_workspace_size(tokens, heads, d, max_seq_len);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, query.options().dtype(at::kByte));
  CheckStatus(hif8_paged_attention_strided(
                  reinterpret_cast<const uint16_t *>(query.data_ptr()), key_cache.data_ptr<uint8_t>(),
                  value_cache.data_ptr<uint8_t>(), block_tables.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                  query_start.data_ptr<int32_t>(), block_tables.size(0), tokens, heads, key_cache.size(2), d,
                  key_cache.size(0), key_cache.size(1), block_stride, block_tables.size(1), max_seq_len,
                  (float)softmax_scale, causal ? 1 : 0, reinterpret_cast<uint16_t *>(out.data_ptr()),
                  ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, Stream(query)),
              "hif8_paged_attention");
  return out;
}

// ---- glue of the synthetic decoder (include/hif8_b200_model.h) ----------

// align: the widest access the kernel makes to the tensor (16: vector loads)
void CheckModelTensor(const at::Tensor &t, const char *name, at::ScalarType dtype, int align = 16) {
  TORCH_CHECK(t.defined() && t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, ", got ", t.scalar_type());
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % align == 0, name, " must be ", align, "-byte aligned");
}

const uint16_t *Bits(const at::Tensor &t) { return reinterpret_cast<const uint16_t *>(t.data_ptr()); }
uint16_t *MutBits(at::Tensor &t) { return reinterpret_cast<uint16_t *>(t.data_ptr()); }

std::tuple<at::Tensor, at::Tensor> ModelRmsnorm(const at::Tensor &x, const std::optional<at::Tensor> &residual,
                                                const at::Tensor &weight, double eps, bool one_plus) {
  CheckModelTensor(x, "x", at::kBFloat16);
  CheckModelTensor(weight, "weight", at::kBFloat16);
  const int64_t dim = x.size(-1), rows = x.numel() / dim;
  TORCH_CHECK(weight.numel() == dim, "weight must have one value per column");
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty_like(x);
  at::Tensor res_out;
  const uint16_t *res_in = nullptr;
  if (residual.has_value()) {
    CheckModelTensor(*residual, "residual", at::kBFloat16);
    TORCH_CHECK(residual->sizes() == x.sizes(), "residual must match x");
    res_in = Bits(*residual);
    res_out = at::empty_like(x);
  }
  CheckStatus(hif8_model_rmsnorm(Bits(x), res_in, res_in ? MutBits(res_out) : nullptr, Bits(weight), (float)eps,
                                 one_plus ? 1 : 0, rows, dim, MutBits(out), Stream(x)),
              "hif8_model_rmsnorm");
  return {out, res_in ? res_out : x};
}

// Decode-step projection with its glue fused into the quantisation prologue
// (hif8_model_glue_linear): kind 1 silu_mul (x = gate_up [m, 2k]), 2
// gate_mul (aux = gate), 3 rmsnorm (aux = residual or None, norm_w).
// Returns (out [m, n] BF16, new residual: x + aux for kind 3 with aux, else x).
std::tuple<at::Tensor, at::Tensor> ModelGlueLinear(const at::Tensor &x, const std::optional<at::Tensor> &aux,
                                                   const std::optional<at::Tensor> &norm_w, int64_t kind, double eps,
                                                   bool one_plus, const at::Tensor &weight,
                                                   const at::Tensor &fixed_scale, const at::Tensor &weight_scale) {
  CheckModelTensor(x, "x", at::kBFloat16);
  CheckModelTensor(weight, "weight", at::kByte, 32);
  CheckModelTensor(fixed_scale, "fixed_scale", at::kFloat, 4);
  CheckModelTensor(weight_scale, "weight_scale", at::kFloat, 4);
  TORCH_CHECK(kind >= 1 && kind <= 3, "glue kind must be 1 (silu_mul), 2 (gate_mul) or 3 (rmsnorm)");
  TORCH_CHECK(weight.dim() == 2, "weight must be 2D");
  const int64_t width = x.size(-1), rows = x.numel() / width;
  const int64_t k = kind == 1 ? width / 2 : width;
  TORCH_CHECK(kind != 1 || width % 2 == 0, "gate_up width must be even");
  TORCH_CHECK(weight.size(1) == k, "weight K ", weight.size(1), " does not match the activation's ", k);
  TORCH_CHECK(fixed_scale.numel() == 1, "fixed_scale must hold one value");
  TORCH_CHECK(weight_scale.numel() == weight.size(0), "weight_scale must hold one value per output channel");
  Hif8GlueArgs g{};
  g.kind = (int)kind;
  g.eps = (float)eps;
  g.one_plus = one_plus ? 1 : 0;
  at::Tensor res_out = x;
  if (aux.has_value()) {
    CheckModelTensor(*aux, "aux", at::kBFloat16);
    TORCH_CHECK(kind != 1, "silu_mul takes no aux tensor");
    TORCH_CHECK(aux->sizes() == x.sizes(), "aux must match x");
    g.aux = Bits(*aux);
    if (kind == 3) {
      res_out = at::empty_like(x);
      g.residual_out = MutBits(res_out);
    }
  } else {
    TORCH_CHECK(kind != 2, "gate_mul needs the gate as aux");
  }
  if (kind == 3) {
    TORCH_CHECK(norm_w.has_value(), "rmsnorm needs norm_w");
    CheckModelTensor(*norm_w, "norm_w", at::kBFloat16);
    TORCH_CHECK(norm_w->numel() == k, "norm_w must have one value per column");
    g.norm_w = Bits(*norm_w);
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto sizes = x.sizes().vec();
  sizes.back() = weight.size(0);
  auto out = at::empty(sizes, x.options());
  CheckStatus(hif8_model_glue_linear(Bits(x), &g, rows, k, weight.data_ptr<uint8_t>(), fixed_scale.data_ptr<float>(),
                                     weight_scale.data_ptr<float>(), weight.size(0), MutBits(out), Stream(x)),
              "hif8_model_glue_linear");
  return {out, res_out};
}

at::Tensor ModelSiluMul(const at::Tensor &gate_up) {
  CheckModelTensor(gate_up, "gate_up", at::kBFloat16, 4);
  const int64_t two_i = gate_up.size(-1), rows = gate_up.numel() / two_i;
  TORCH_CHECK(two_i % 4 == 0, "gate_up width must be a multiple of 4");
  c10::cuda::CUDAGuard guard(gate_up.device());
  auto sizes = gate_up.sizes().vec();
  sizes.back() = two_i / 2;
  auto out = at::empty(sizes, gate_up.options());
  CheckStatus(hif8_model_silu_mul(Bits(gate_up), rows, two_i / 2, MutBits(out), Stream(gate_up)),
              "hif8_model_silu_mul");
  return out;
}

at::Tensor ModelGateMul(const at::Tensor &x, const at::Tensor &gate) {
  CheckModelTensor(x, "x", at::kBFloat16, 2);
  CheckModelTensor(gate, "gate", at::kBFloat16, 2);
  TORCH_CHECK(x.numel() == gate.numel(), "gate must match x");
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty_like(x);
  CheckStatus(hif8_model_gate_mul(Bits(x), Bits(gate), x.numel(), MutBits(out), Stream(x)), "hif8_model_gate_mul");
  return out;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> ModelAttnPrep(
    const at::Tensor &qkv, const at::Tensor &positions, const at::Tensor &q_norm_w, const at::Tensor &k_norm_w,
    int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t rotary_dim, double eps, double rope_theta) {
  CheckModelTensor(qkv, "qkv", at::kBFloat16, 2);
  CheckModelTensor(positions, "positions", at::kInt, 4);
  CheckModelTensor(q_norm_w, "q_norm_w", at::kBFloat16, 2);
  CheckModelTensor(k_norm_w, "k_norm_w", at::kBFloat16, 2);
  const int64_t tokens = qkv.size(0);
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(1) == (2 * heads + 2 * kv_heads) * head_dim, "qkv must be [tokens, "
              "(2 heads + 2 kv_heads) head_dim]");
  TORCH_CHECK(positions.numel() == tokens, "positions must have one entry per token");
  c10::cuda::CUDAGuard guard(qkv.device());
  auto q = at::empty({tokens, heads, head_dim}, qkv.options());
  auto gate = at::empty({tokens, heads * head_dim}, qkv.options());
  auto k = at::empty({tokens, kv_heads, head_dim}, qkv.options());
  auto v = at::empty({tokens, kv_heads, head_dim}, qkv.options());
  CheckStatus(hif8_model_attn_prep(Bits(qkv), tokens, (int)heads, (int)kv_heads, (int)head_dim, (int)rotary_dim,
                                   positions.data_ptr<int32_t>(), Bits(q_norm_w), Bits(k_norm_w), (float)eps,
                                   (float)rope_theta, MutBits(q), MutBits(gate), MutBits(k), MutBits(v), Stream(qkv)),
              "hif8_model_attn_prep");
  return {q, gate, k, v};
}

at::Tensor ModelGdn(const at::Tensor &proj, int64_t T, int64_t hk, int64_t hv, const at::Tensor &conv_w,
                    const at::Tensor &a_log, const at::Tensor &dt_bias, const at::Tensor &norm_w,
                    at::Tensor &conv_state, at::Tensor &rec_state, double eps) {
  CheckModelTensor(proj, "proj", at::kBFloat16, 2);
  CheckModelTensor(conv_w, "conv_w", at::kBFloat16, 2);
  CheckModelTensor(a_log, "a_log", at::kFloat, 4);
  CheckModelTensor(dt_bias, "dt_bias", at::kFloat, 4);
  CheckModelTensor(norm_w, "norm_w", at::kBFloat16, 2);
  CheckModelTensor(conv_state, "conv_state", at::kFloat, 4);
  CheckModelTensor(rec_state, "rec_state", at::kFloat, 4);
  const int64_t channels = 2 * hk * 128 + hv * 128;
  TORCH_CHECK(proj.dim() == 2 && proj.size(1) == channels + hv * 128 + 2 * hv, "proj must be [batch * T, "
              "2 hk 128 + 2 hv 128 + 2 hv]");
  TORCH_CHECK(T > 0 && proj.size(0) % T == 0, "proj rows must be a multiple of T");
  const int64_t batch = proj.size(0) / T;
  TORCH_CHECK(conv_w.numel() == channels * 4, "conv_w must be [channels, 4]");
  TORCH_CHECK(conv_state.numel() == batch * hv * 3 * 128 * 3, "conv_state must be [batch, hv, 3, 128, 3]");
  TORCH_CHECK(rec_state.numel() == batch * hv * 128 * 128, "rec_state must be [batch, hv, 128, 128]");
  c10::cuda::CUDAGuard guard(proj.device());
  auto out = at::empty({proj.size(0), hv * 128}, proj.options());
  Hif8GdnArgs args{};
  args.proj = Bits(proj);
  args.proj_stride = proj.size(1);
  args.T = (int)T;
  args.hk = (int)hk;
  args.hv = (int)hv;
  args.key_dim = 128;
  args.value_dim = 128;
  args.conv_w = Bits(conv_w);
  args.a_log = a_log.data_ptr<float>();
  args.dt_bias = dt_bias.data_ptr<float>();
  args.norm_w = Bits(norm_w);
  args.conv_state = conv_state.data_ptr<float>();
  args.rec_state = rec_state.data_ptr<float>();
  args.out = MutBits(out);
  args.eps = (float)eps;
  CheckStatus(hif8_model_gdn(&args, batch, Stream(proj)), "hif8_model_gdn");
  return out;
}

// Tensor-parallel partial product of a row-parallel static linear: x
// (FP16/BF16 [M, K], this rank's input columns) statically quantised with
// input_scale, times this rank's weight columns, as FP32 [M, N] without
// rounding (the ranks' partials are summed before the one BF16 rounding).
// M <= 4: one fused quant + GEMV launch; larger M: static quant, then the
// GEMV / tcgen05 GEMM with FP32 output.
at::Tensor Hif8LinearPartialF32(const at::Tensor &x_in, const at::Tensor &weight_in, const at::Tensor &input_scale_in,
                                const at::Tensor &weight_scale_in) {
  // an internal operator: any CUDA layout is accepted and made contiguous
  // (the kernels pick their vector paths by alignment)
  for (const at::Tensor *t : {&x_in, &weight_in, &input_scale_in, &weight_scale_in})
    TORCH_CHECK(t->defined() && t->is_cuda(), "linear_partial_f32 operands must be CUDA tensors");
  const at::Tensor x = x_in.contiguous(), weight = weight_in.contiguous();
  const at::Tensor input_scale = input_scale_in.contiguous(), weight_scale = weight_scale_in.contiguous();
  TORCH_CHECK(x.scalar_type() == at::ScalarType::Half || x.scalar_type() == at::ScalarType::BFloat16,
              "x must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte && weight.dim() == 2, "weight must be uint8 [N, K]");
  TORCH_CHECK(input_scale.scalar_type() == at::ScalarType::Float && input_scale.numel() == 1,
              "input_scale must be one float32 value");
  TORCH_CHECK(weight_scale.scalar_type() == at::ScalarType::Float && weight_scale.numel() == weight.size(0),
              "weight_scale must contain one float32 value per output channel");
  TORCH_CHECK(x.size(-1) == weight.size(1), "x and weight K dimensions differ");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t k = x.size(-1), m = x.numel() / k, n = weight.size(0);
  auto out = at::empty({m, n}, x.options().dtype(at::kFloat));
  if (m == 0) return out;
  const int x_dtype = DtypeCode(x.scalar_type());
  // fused quant + GEMV for the rows the scheme fuses (<= 4): beyond that
  // every CTA would quantise all rows of its K slice, where one quant launch
  // does it once
  if (m <= 4) {
    CheckStatus(hif8_static_fused_linear_partial_f32(x.data_ptr(), x_dtype, weight.data_ptr<uint8_t>(),
                                                     input_scale.data_ptr<float>(), weight_scale.data_ptr<float>(), m,
                                                     n, k, out.data_ptr<float>(), Stream(x)),
                "hif8_static_fused_linear_partial_f32");
    return out;
  }
  auto data = at::empty({m, k}, x.options().dtype(at::kByte));
  auto row_scale = at::empty({m}, x.options().dtype(at::kFloat));
  CheckStatus(hif8_static_quant(x.data_ptr(), x_dtype, m, k, input_scale.data_ptr<float>(), 1,
                                data.data_ptr<uint8_t>(), row_scale.data_ptr<float>(), Stream(x)),
              "hif8_static_quant");
  const size_t ws_bytes = soft_hif8_gemm_workspace_size(m, n, k);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({(int64_t)ws_bytes}, x.options().dtype(at::kByte));
  CheckStatus(hif8_linear_partial_f32(data.data_ptr<uint8_t>(), weight.data_ptr<uint8_t>(),
                                      row_scale.data_ptr<float>(), weight_scale.data_ptr<float>(), m, n, k,
                                      out.data_ptr<float>(), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, Stream(x)),
              "hif8_linear_partial_f32");
  return out;
}

// The static scheme's apply (reference scheme.py:174-211) as one operator:
// the routing between the fused quant + linear (rows <= fused_max_rows) and
// quant then linear happens here, so a projection costs one dispatch.  The
// checks are the ones the two reference operators make, with their messages.
at::Tensor Hif8StaticLinear(const at::Tensor &x_in, const at::Tensor &weight, const at::Tensor &input_scale,
                            const at::Tensor &weight_scale, const std::optional<at::Tensor> &bias,
                            int64_t fused_max_rows) {
  TORCH_CHECK(x_in.defined() && x_in.is_cuda(), "x must be a CUDA tensor");
  TORCH_CHECK(x_in.scalar_type() == at::ScalarType::Half || x_in.scalar_type() == at::ScalarType::BFloat16,
              "x must have dtype torch.float16 or torch.bfloat16");
  TORCH_CHECK(x_in.dim() >= 2, "x must have shape [..., K]");
  // a contiguous view at any 16-byte aligned offset is used in place; any
  // other layout is copied (to an aligned allocation, so the kernels take
  // the same vector paths -- and give the same bits -- as for an owned tensor)
  const bool in_place = x_in.is_contiguous() && (reinterpret_cast<uintptr_t>(x_in.data_ptr()) & 15u) == 0;
  const at::Tensor x = in_place ? x_in : x_in.contiguous().clone();
  CheckCudaTensor(weight, "weight");
  CheckCudaTensor(input_scale, "fixed_scale");
  CheckCudaTensor(weight_scale, "channel_scale");
  TORCH_CHECK(weight.scalar_type() == at::ScalarType::Byte, "weight must have dtype torch.uint8");
  TORCH_CHECK(weight.dim() == 2, "weight must have shape [N, K]");
  TORCH_CHECK(input_scale.scalar_type() == at::ScalarType::Float, "fixed_scale must have dtype torch.float32");
  TORCH_CHECK(input_scale.numel() == 1, "fixed_scale must have shape [1]");
  TORCH_CHECK(weight_scale.scalar_type() == at::ScalarType::Float, "channel_scale must have dtype torch.float32");
  CheckPositiveDimensions(x, "activation");
  CheckPositiveDimensions(weight, "weight");
  const int64_t k = x.size(-1), m = x.numel() / k, n = weight.size(0);
  TORCH_CHECK(weight.size(1) == k, "activation and weight K dimensions differ: ", k, " != ", weight.size(1));
  TORCH_CHECK(weight_scale.numel() == n, "channel_scale must contain one value per output channel");
  CheckFitsUint32(m, "M");
  CheckFitsUint32(n, "N");
  CheckFitsUint32(k, "K");
  const auto device = x.device();
  CheckSameDevice(weight, device, "weight");
  CheckSameDevice(input_scale, device, "fixed_scale");
  CheckSameDevice(weight_scale, device, "channel_scale");
  const void *bias_ptr = nullptr;
  int bias_dtype = HIF8_DTYPE_NONE;
  if (bias.has_value()) {
    CheckCudaTensor(*bias, "bias");
    CheckSameDevice(*bias, device, "bias");
    TORCH_CHECK(bias->dim() == 1, "bias must have shape [N]");
    TORCH_CHECK(bias->numel() == n, "bias must contain N values");
    TORCH_CHECK(bias->scalar_type() == at::ScalarType::Half || bias->scalar_type() == at::ScalarType::BFloat16,
                "bias must have dtype torch.float16 or torch.bfloat16");
    bias_ptr = bias->data_ptr();
    bias_dtype = DtypeCode(bias->scalar_type());
  }
  c10::cuda::CUDAGuard guard(device);
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = n;
  auto out = at::empty(out_shape, x.options());
  const int fused = (int)std::max<int64_t>(0, std::min<int64_t>(fused_max_rows, 4));
  const size_t ws_bytes = hif8_static_linear_workspace_size(m, n, k, fused);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({(int64_t)ws_bytes}, x.options().dtype(at::kByte));
  const int dtype = DtypeCode(x.scalar_type());
  CheckStatus(hif8_static_linear(x.data_ptr(), dtype, weight.data_ptr<uint8_t>(), input_scale.data_ptr<float>(),
                                 weight_scale.data_ptr<float>(), bias_ptr, bias_dtype, dtype, m, n, k, fused,
                                 out.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, Stream(x)),
              "hif8_static_linear");
  return out;
}

std::tuple<at::Tensor, at::Tensor> ModelPeerAllreduceRmsnorm(const at::Tensor &local,
                                                             const std::optional<at::Tensor> &residual,
                                                             const at::Tensor &weight, const at::Tensor &peer_buf,
                                                             at::Tensor &counter, at::Tensor &error, int64_t max_rows,
                                                             int64_t rank, int64_t world, int64_t slot, double eps,
                                                             bool one_plus, int64_t timeout_ns) {
  TORCH_CHECK(local.scalar_type() == at::kFloat || local.scalar_type() == at::kBFloat16,
              "local must be a float32 or bfloat16 partial");
  CheckModelTensor(local, "local", local.scalar_type());
  CheckModelTensor(weight, "weight", at::kBFloat16);
  CheckModelTensor(peer_buf, "peer_buf", at::kLong);
  CheckModelTensor(counter, "counter", at::kInt, 4);
  CheckModelTensor(error, "error", at::kInt, 4);
  TORCH_CHECK(peer_buf.numel() == world, "peer_buf must hold one buffer per rank");
  const int64_t dim = local.size(-1), rows = local.numel() / dim;
  c10::cuda::CUDAGuard guard(local.device());
  auto out = at::empty(local.sizes(), local.options().dtype(at::kBFloat16));
  auto res_out = at::empty(local.sizes(), local.options().dtype(at::kBFloat16));
  Hif8PeerArgs a{};
  a.local = local.data_ptr();
  a.local_dtype = local.scalar_type() == at::kFloat ? HIF8_DTYPE_F32 : HIF8_DTYPE_BF16;
  if (residual.has_value()) {
    CheckModelTensor(*residual, "residual", at::kBFloat16);
    TORCH_CHECK(residual->sizes() == local.sizes(), "residual must match local");
    a.residual = Bits(*residual);
  }
  a.weight = Bits(weight);
  a.out = MutBits(out);
  a.residual_out = MutBits(res_out);
  a.peer_buf = reinterpret_cast<uint8_t *const *>(peer_buf.data_ptr<int64_t>());
  a.epoch_counter = reinterpret_cast<uint32_t *>(counter.data_ptr<int32_t>());
  a.error = error.data_ptr<int32_t>();
  a.rows = rows;
  a.dim = dim;
  a.max_rows = max_rows;
  a.rank = (int)rank;
  a.world = (int)world;
  a.slot = (int)slot;
  a.one_plus = one_plus ? 1 : 0;
  a.eps = (float)eps;
  a.timeout_ns = (uint64_t)timeout_ns;
  CheckStatus(hif8_model_peer_allreduce_rmsnorm(&a, Stream(local)), "hif8_model_peer_allreduce_rmsnorm");
  return {out, res_out};
}

// The all-reduced sum of the ranks' partials (no norm): the same push
// exchange with a null weight.
at::Tensor ModelPeerAllreduce(const at::Tensor &local, const at::Tensor &peer_buf, at::Tensor &counter,
                              at::Tensor &error, int64_t max_rows, int64_t rank, int64_t world, int64_t slot,
                              int64_t timeout_ns) {
  TORCH_CHECK(local.scalar_type() == at::kFloat || local.scalar_type() == at::kBFloat16,
              "local must be a float32 or bfloat16 partial");
  CheckModelTensor(local, "local", local.scalar_type());
  CheckModelTensor(peer_buf, "peer_buf", at::kLong);
  CheckModelTensor(counter, "counter", at::kInt, 4);
  CheckModelTensor(error, "error", at::kInt, 4);
  TORCH_CHECK(peer_buf.numel() == world, "peer_buf must hold one buffer per rank");
  const int64_t dim = local.size(-1), rows = local.numel() / dim;
  c10::cuda::CUDAGuard guard(local.device());
  auto out = at::empty(local.sizes(), local.options().dtype(at::kBFloat16));
  Hif8PeerArgs a{};
  a.local = local.data_ptr();
  a.local_dtype = local.scalar_type() == at::kFloat ? HIF8_DTYPE_F32 : HIF8_DTYPE_BF16;
  a.out = MutBits(out);
  a.peer_buf = reinterpret_cast<uint8_t *const *>(peer_buf.data_ptr<int64_t>());
  a.epoch_counter = reinterpret_cast<uint32_t *>(counter.data_ptr<int32_t>());
  a.error = error.data_ptr<int32_t>();
  a.rows = rows;
  a.dim = dim;
  a.max_rows = max_rows;
  a.rank = (int)rank;
  a.world = (int)world;
  a.slot = (int)slot;
  a.timeout_ns = (uint64_t)timeout_ns;
  CheckStatus(hif8_model_peer_allreduce_rmsnorm(&a, Stream(local)), "hif8_model_peer_allreduce_rmsnorm");
  return out;
}

at::Tensor Hif8KvGatherDecode(const at::Tensor &cache, const at::Tensor &block_tables, const at::Tensor &seq_lens,
                              const at::Tensor &out_start, int64_t total_rows, int64_t max_seq_len) {
  CheckCudaTensor(cache, "cache");
  CheckCudaTensor(block_tables, "block_tables");
  CheckCudaTensor(seq_lens, "seq_lens");
  CheckCudaTensor(out_start, "out_start");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 4, "cache must be uint8 [blocks, block_size, heads, D + 4]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  out_start.scalar_type() == at::kInt,
              "block_tables/seq_lens/out_start must be int32");
  c10::cuda::CUDAGuard guard(cache.device());
  const int64_t heads = cache.size(2), d = cache.size(3) - 4;
  auto out = at::empty({total_rows, heads, d}, cache.options().dtype(at::kBFloat16));
  if (total_rows == 0) return out;
  CheckStatus(hif8_kv_gather_decode(cache.data_ptr<uint8_t>(), block_tables.data_ptr<int32_t>(),
                                    seq_lens.data_ptr<int32_t>(), out_start.data_ptr<int32_t>(), block_tables.size(0),
                                    heads, d, cache.size(0), cache.size(1), block_tables.size(1), max_seq_len,
                                    reinterpret_cast<uint16_t *>(out.data_ptr()), Stream(cache)),
              "hif8_kv_gather_decode");
  return out;
}

std::vector<int64_t> RowScaleShape(const at::Tensor &x) {
  return {x.dim() >= 1 && x.size(-1) > 0 ? x.numel() / x.size(-1) : 1};
}

}  // namespace

TORCH_LIBRARY(vllm_ascend_hif8, m) {
  m.def("hif8_dynamic_quant(Tensor x) -> (Tensor, Tensor)");
  m.def("hif8_static_quant(Tensor x, Tensor fixed_scale) -> (Tensor, Tensor)");
  m.def("hif8_scaled_decode(Tensor data, Tensor scale) -> Tensor");
  m.def("soft_hif8_gemv(Tensor activation, Tensor weight, Tensor token_scale, Tensor channel_scale, Tensor? bias, "
        "ScalarType output_dtype) -> Tensor");
  m.def("soft_hif8_gemm(Tensor activation, Tensor weight, Tensor token_scale, Tensor channel_scale, Tensor? bias, "
        "ScalarType output_dtype) -> Tensor");
  m.def("soft_hif8_fused_gemm(Tensor activation, Tensor weight, Tensor channel_scale, Tensor? bias, "
        "ScalarType output_dtype) -> Tensor");
  m.def("soft_hif8_static_fused_gemm(Tensor activation, Tensor weight, Tensor fixed_scale, Tensor channel_scale, "
        "Tensor? bias, ScalarType output_dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(vllm_ascend_hif8, CUDA, m) {
  m.impl("hif8_dynamic_quant", &Hif8DynamicQuant);
  m.impl("hif8_static_quant", &Hif8StaticQuant);
  m.impl("hif8_scaled_decode", &Hif8ScaledDecode);
  m.impl("soft_hif8_gemv", &SoftHif8Gemv);
  m.impl("soft_hif8_gemm", &SoftHif8Gemm);
  m.impl("soft_hif8_fused_gemm", &SoftHif8FusedGemm);
  m.impl("soft_hif8_static_fused_gemm", &SoftHif8StaticFusedGemm);
}

TORCH_LIBRARY_IMPL(vllm_ascend_hif8, Meta, m) {
  m.impl("hif8_static_quant", [](const at::Tensor &x, const at::Tensor &) -> std::tuple<at::Tensor, at::Tensor> {
    return {at::empty_like(x, x.options().dtype(at::kByte)), at::empty(RowScaleShape(x), x.options().dtype(at::kFloat))};
  });
  m.impl("hif8_scaled_decode", [](const at::Tensor &data, const at::Tensor &) -> at::Tensor {
    return at::empty_like(data, data.options().dtype(at::kBFloat16));
  });
  auto linear_meta = [](const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &, const at::Tensor &,
                        const std::optional<at::Tensor> &, at::ScalarType output_dtype) -> at::Tensor {
    return at::empty({activation.size(0), weight.size(0)}, activation.options().dtype(output_dtype));
  };
  m.impl("soft_hif8_gemv", linear_meta);
  m.impl("soft_hif8_gemm", linear_meta);
  m.impl("soft_hif8_static_fused_gemm", linear_meta);
  m.impl("hif8_dynamic_quant", [](const at::Tensor &x) -> std::tuple<at::Tensor, at::Tensor> {
    return {at::empty_like(x, x.options().dtype(at::kByte)),
            at::empty({x.numel() / x.size(-1)}, x.options().dtype(at::kFloat))};
  });
  m.impl("soft_hif8_fused_gemm", [](const at::Tensor &activation, const at::Tensor &weight, const at::Tensor &,
                                    const std::optional<at::Tensor> &, at::ScalarType output_dtype) -> at::Tensor {
    return at::empty({activation.size(0), weight.size(0)}, activation.options().dtype(output_dtype));
  });
}

TORCH_LIBRARY(hif8_b200, m) {
  m.def("kv_cache_write(Tensor key, Tensor value, Tensor key_scale, Tensor value_scale, Tensor slot_mapping, "
        "Tensor(a!) key_cache, Tensor(b!) value_cache, Tensor(c!)? bad_slots=None) -> ()");
  m.def("paged_attention(Tensor query, Tensor key_cache, Tensor value_cache, Tensor block_tables, Tensor seq_lens, "
        "Tensor query_start, int max_seq_len, float softmax_scale, bool causal=True) -> Tensor");
  m.def("kv_gather_decode(Tensor cache, Tensor block_tables, Tensor seq_lens, Tensor out_start, int total_rows, "
        "int max_seq_len) -> Tensor");
  m.def("embedding_gather(Tensor weight, Tensor weight_scale, Tensor ids, Tensor(a!)? bad_ids=None) -> Tensor");
  // glue of the synthetic decoder
  m.def("rmsnorm(Tensor x, Tensor? residual, Tensor weight, float eps, bool one_plus) -> (Tensor, Tensor)");
  m.def("silu_mul(Tensor gate_up) -> Tensor");
  m.def("glue_linear(Tensor x, Tensor? aux, Tensor? norm_w, int kind, float eps, bool one_plus, Tensor weight, "
        "Tensor fixed_scale, Tensor weight_scale) -> (Tensor, Tensor)");
  m.def("gate_mul(Tensor x, Tensor gate) -> Tensor");
  m.def("attn_prep(Tensor qkv, Tensor positions, Tensor q_norm_w, Tensor k_norm_w, int heads, int kv_heads, "
        "int head_dim, int rotary_dim, float eps, float rope_theta) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("gdn(Tensor proj, int T, int hk, int hv, Tensor conv_w, Tensor a_log, Tensor dt_bias, Tensor norm_w, "
        "Tensor(a!) conv_state, Tensor(b!) rec_state, float eps) -> Tensor");
  m.def("peer_allreduce_rmsnorm(Tensor local, Tensor? residual, Tensor weight, Tensor peer_buf, Tensor(a!) counter, "
        "Tensor(b!) error, int max_rows, int rank, int world, int slot, float eps, bool one_plus, int timeout_ns) "
        "-> (Tensor, Tensor)");
  m.def("peer_allreduce(Tensor local, Tensor peer_buf, Tensor(a!) counter, Tensor(b!) error, int max_rows, int rank, "
        "int world, int slot, int timeout_ns) -> Tensor");
  m.def("linear_partial_f32(Tensor x, Tensor weight, Tensor input_scale, Tensor weight_scale) -> Tensor");
  m.def("static_linear(Tensor x, Tensor weight, Tensor input_scale, Tensor weight_scale, Tensor? bias=None, "
        "int fused_max_rows=4) -> Tensor");
}

TORCH_LIBRARY_IMPL(hif8_b200, Meta, m) {
  m.impl("static_linear", [](const at::Tensor &x, const at::Tensor &weight, const at::Tensor &, const at::Tensor &,
                             const std::optional<at::Tensor> &, int64_t) -> at::Tensor {
    std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
    shape.back() = weight.size(0);
    return at::empty(shape, x.options());
  });
}

TORCH_LIBRARY_IMPL(hif8_b200, CUDA, m) {
  m.impl("kv_cache_write", &Hif8KvCacheWrite);
  m.impl("paged_attention", &Hif8PagedAttention);
  m.impl("kv_gather_decode", &Hif8KvGatherDecode);
  m.impl("embedding_gather", &Hif8EmbeddingGather);
  m.impl("rmsnorm", &ModelRmsnorm);
  m.impl("silu_mul", &ModelSiluMul);
  m.impl("glue_linear", &ModelGlueLinear);
  m.impl("gate_mul", &ModelGateMul);
  m.impl("attn_prep", &ModelAttnPrep);
  m.impl("gdn", &ModelGdn);
  m.impl("peer_allreduce_rmsnorm", &ModelPeerAllreduceRmsnorm);
  m.impl("peer_allreduce", &ModelPeerAllreduce);
  m.impl("linear_partial_f32", &Hif8LinearPartialF32);
  m.impl("static_linear", &Hif8StaticLinear);
}
