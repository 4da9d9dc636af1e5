// Shared device/host helpers of the hif8_b200 kernels (sm_100a).
//
// HiFloat8 (HiF8) byte layout, Ascend order (reference
// src/vllm_ascend_hif8/codec.py:15-82): bit 7 = sign; magnitude 0 = zero,
// 0x80 = NaN, 0x6F/0xEF = +-Inf; codes 1..7 are 2^-22..2^-16; normal
// exponent classes |e|<=3 (3 mantissa bits, bases 0x08..0x38), 4..7 (2 bits,
// 0x40/0x50), 8..15 (1 bit, 0x60/0x70).  Every finite code is exactly a BF16.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/hif8_b200.h"

#define HIF8_HD __host__ __device__ __forceinline__

namespace hif8 {

// ----------------------------------------------------------------- codec --

// Lower seven bits of a finite normal value 2^e * (1 + i / 2^mb)
// (codec.py:27-49).
HIF8_HD constexpr uint32_t normal_code(int e, int i) {
  return (e >= -3 && e <= 3)
             ? (uint32_t)((e == 0 ? 0x08 : e == 1 ? 0x10 : e == -1 ? 0x18 : e == 2 ? 0x20
                           : e == 3 ? 0x28 : e == -2 ? 0x30 : 0x38) + i)
         : (e >= 4 && e <= 7)   ? (uint32_t)(0x40 + (e - 4) * 4 + i)
         : (e <= -4 && e >= -7) ? (uint32_t)(0x50 + (-e - 4) * 4 + i)
         : (e >= 8)             ? (uint32_t)(0x60 + (e - 8) * 2 + i)
                                : (uint32_t)(0x70 + (-e - 8) * 2 + i);
}

HIF8_HD constexpr int mantissa_bits(int e) {
  return (e <= 3 && e >= -3) ? 3 : (e <= 7 && e >= -7) ? 2 : 1;
}

// Magnitude code of the FP32 grid value (exponent field E, top-4 mantissa
// bits t), nearest with ties away from zero -- the rule that generates the
// 4096-entry table of torch_codec.py:19-29.  An FP32 value encodes exactly
// like its truncation to this grid because no code has more than 3 mantissa
// bits, so the 4th bit alone decides every tie.
HIF8_HD constexpr uint32_t encode_grid(uint32_t idx) {
  const uint32_t E = idx >> 4, t = idx & 15u;
  if (E == 255u) return t == 0 ? 0x6Fu : 0x00u;  // Inf -> 0x6F, NaN -> 0x80 & 0x7F
  if (E == 0u) return 0u;                         // FP32 denormals underflow
  int e = (int)E - 127;
  if (e < -23) return 0u;                         // below the 2^-23 underflow tie
  if (e == -23) return 1u;                        // [2^-23, 2^-22) -> 2^-22
  if (e <= -16) {                                 // between powers of two 2^-22..2^-15
    if (t < 8u) return (uint32_t)(e + 23);
    return e + 1 <= -16 ? (uint32_t)(e + 24) : normal_code(-15, 0);
  }
  if (e > 15) return 0x6Fu;                       // overflow -> Inf
  const int mb = mantissa_bits(e);
  int i = (int)(t >> (4 - mb)) + (int)((t >> (3 - mb)) & 1u);
  if (i == (1 << mb)) {
    i = 0;
    e += 1;
  }
  if (e > 15) return 0x6Fu;
  return normal_code(e, i);  // normal_code(15, 1) == 0x6F: the overflow tie
}

// Static-saturating signed encode, indexed by the top 13 bits of an FP32
// (sign, exponent, top-4 mantissa): finite overflow saturates to +-0x6E
// (calibration.py:139-158, tablegen.py:40-49); E == 255 yields Inf / NaN.
HIF8_HD constexpr uint8_t static_encode13(uint32_t i13) {
  const uint32_t sign = (i13 >> 12) & 1u;
  const uint32_t idx = i13 & 0xFFFu;
  if ((idx >> 4) == 255u) return (idx & 15u) == 0 ? (uint8_t)(0x6Fu | (sign << 7)) : (uint8_t)0x80u;
  uint32_t mag = encode_grid(idx);
  if (mag == 0x6Fu) mag = 0x6Eu;
  return mag == 0 ? (uint8_t)0 : (uint8_t)(mag | (sign << 7));
}

// BF16 payload of a byte (codec.py:106-145); NaN -> 0x7FC0.
HIF8_HD constexpr uint32_t decode_bf16(uint32_t b) {
  if (b == 0x80u) return 0x7FC0u;
  const uint32_t sign = (b & 0x80u) << 8;
  const uint32_t m = b & 0x7Fu;
  if (m == 0) return sign;
  if (m == 0x6Fu) return sign | 0x7F80u;
  uint32_t ef = 0, fr = 0;
  if (m <= 7) {
    ef = 104 + m;
  } else if (m <= 63) {
    const uint32_t g = m >> 3;
    ef = g == 1 ? 127 : g == 2 ? 128 : g == 3 ? 126 : g == 4 ? 129 : g == 5 ? 130 : g == 6 ? 125 : 124;
    fr = (m & 7u) << 4;
  } else if (m <= 79) {
    ef = 131 + ((m - 64) >> 2);
    fr = (m & 3u) << 5;
  } else if (m <= 95) {
    ef = 123 - ((m - 80) >> 2);
    fr = (m & 3u) << 5;
  } else if (m <= 110) {
    ef = 135 + ((m - 96) >> 1);
    fr = (m & 1u) << 6;
  } else {
    ef = 119 - ((m - 112) >> 1);
    fr = (m & 1u) << 6;
  }
  return sign | (ef << 7) | fr;
}

struct alignas(16) Table13 {
  uint8_t v[8192];
};
struct alignas(16) Table256 {
  uint32_t v[256];
};

HIF8_HD constexpr Table13 make_static_encode_table() {
  Table13 t{};
  for (uint32_t i = 0; i < 8192u; ++i) t.v[i] = static_encode13(i);
  return t;
}

// Decoded value as FP32 bits (BF16 payload << 16).
HIF8_HD constexpr Table256 make_decode_table_f32() {
  Table256 t{};
  for (uint32_t b = 0; b < 256u; ++b) t.v[b] = decode_bf16(b) << 16;
  return t;
}

// Device copies of the tables (one per translation unit that uses them).
static __device__ const Table13 g_static_encode = make_static_encode_table();
static __device__ const Table256 g_decode_f32 = make_decode_table_f32();

// ---------------------------------------------------- float conversions --

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}
template <int kDtype>
__device__ __forceinline__ float half_bits_to_f32(uint32_t h) {
  if constexpr (kDtype == HIF8_DTYPE_BF16) return bf16_bits_to_f32(h);
  else return f16_bits_to_f32(h);
}

// Nearest-even FP32 -> BF16 with canonical NaN 0x7FC0 (the c10::BFloat16
// rule): add 0x7FFF plus the lowest kept bit, truncate.
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

__device__ __forceinline__ uint32_t f32_to_f16_bits(float v) {
  return (uint32_t)__half_as_ushort(__float2half_rn(v));
}

template <int kDtype>
__device__ __forceinline__ uint32_t f32_to_half_bits(float v) {
  if constexpr (kDtype == HIF8_DTYPE_BF16) return f32_to_bf16_bits(v);
  else return f32_to_f16_bits(v);
}

// Elementwise producers shared by the model glue kernels and the GEMV
// prologue that fuses them (one definition, so both round identically).
__device__ __forceinline__ float glue_silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float glue_sigmoid(float x) { return 1.f / (1.f + __expf(-x)); }

// --------------------------------------------------------- error plumbing --

void set_last_error(cudaError_t err);
int check_launch();

inline int div_up(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

int num_sms();

// Raise a kernel's dynamic shared-memory limit once per device (the call is
// skipped when the limit already suffices, so launches under CUDA-graph
// capture issue no attribute calls after the first eager launch).
int ensure_smem_limit(const void *kernel, size_t bytes);

// Argument checks of hif8_paged_attention (null pointers, non-positive or
// inconsistent sizes, GQA group above 16): HIF8_OK or
// HIF8_ERR_INVALID_ARGUMENT.  Shared by every attention entry point so they
// report the same status for the same bad call.
int paged_attention_args_status(const void *query, const void *key_cache, const void *value_cache,
                                const void *block_tables, const void *seq_lens, const void *query_start,
                                const void *out, int64_t batch, int64_t num_tokens, int64_t num_heads,
                                int64_t kv_heads, int64_t head_size, int64_t num_blocks, int64_t block_size,
                                int64_t max_blocks, int64_t max_seq_len);

// ------------------------------------------- programmatic dependent launch --
// The decode-path kernels are launched with the programmatic stream
// serialization attribute, so the next kernel of the stream is launched as
// soon as this one's CTAs have exited, overlapping its launch with the
// completion of this one.  Every such kernel calls pdl_wait() before it reads
// anything an earlier kernel of the stream may have written and before its
// first global write: the wait returns once the preceding kernel has
// completed and its writes are visible (immediately for an ordinary launch).
// Work before the wait touches only constant tables and shared memory, or
// issues L2 prefetches (L2 is the coherence point, so a prefetch never
// yields a stale value).  Only small grids signal their dependents early
// (griddepcontrol.launch_dependents, at their start): the vectorised static
// quant and the decoder's glue kernels at small batch leave most SMs idle,
// so the following linear's CTAs launch there and build their tables before
// they wait for the signalling grid's completion (the configs[1] step 358.9
// -> 354.7 us).  For the GEMV, which fills every
// SM, an early signal made the sweep 5 % slower as a CUDA graph, while the
// implicit signal at exit made it 2 % faster than ordinary launches.

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// False when the environment sets HIF8_DISABLE_PDL=1 (read once).
bool pdl_enabled();

// Launch `kernel` on `stream`, with the programmatic serialization attribute
// unless disabled; returns a HIF8_* status.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    set_last_error(err);
    return HIF8_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace hif8
