// Shared declarations of the HiF8 linear kernels (split-K GEMV and the
// tcgen05 prefill GEMM).
#pragma once

#include "hif8_common.cuh"

namespace hif8 {

// Producer of the fused linear's activation, applied in the prologue before
// the static quantisation (decode-step glue of the synthetic decoder).
constexpr int kGlueNone = 0;
constexpr int kGlueSiluMul = 1;  // silu(x[:, :k]) * x[:, k:2k], x row stride 2k
constexpr int kGlueGateMul = 2;  // x * sigmoid(aux)
constexpr int kGlueRmsNorm = 3;  // RMSNorm(x + aux) * (one_plus ? 1 + w : w); aux may be null

struct GlueArgs {
  int kind = kGlueNone;
  const uint16_t *aux = nullptr;     // gate (kGlueGateMul) / residual (kGlueRmsNorm)
  uint16_t *residual_out = nullptr;  // kGlueRmsNorm with aux: x + aux (BF16), written by CTA 0
  const uint16_t *norm_w = nullptr;  // kGlueRmsNorm: [k]
  float eps = 0.f;
  int one_plus = 0;
};

struct GemvArgs {
  const void *a;          // [M, K]: HiF8 bytes, or FP16/BF16 for the fused quant path
  const uint8_t *w;       // [N, K]
  const float *ts;        // [M] (or [1] with ts_stride 0)
  const float *cs;        // [N]
  const void *bias;       // [N] or null
  void *out;              // [M, N]
  int m, n, k;
  int kc;                 // K range per CTA (multiple of 64)
  int bias_dtype;
  int ts_stride;          // 1: one token scale per row; 0: one shared fixed scale
  GlueArgs glue;          // fused activation producer (BF16 glue kernels only)
};

bool hif8_gemm_tc_supported(int64_t m, int64_t n, int64_t k);
size_t hif8_gemm_tc_workspace(int64_t m, int64_t n, int64_t k);
// a_dtype: HIF8_DTYPE_NONE for HiF8 activation bytes (args.ts per row), or
// HIF8_DTYPE_BF16 / HIF8_DTYPE_F16 for activations statically quantised in
// the GEMM's operand pass with the fixed scale args.ts[0] (ts_stride 0).
int hif8_gemm_tc(const GemvArgs &args, int output_dtype, void *workspace, size_t workspace_bytes,
                 cudaStream_t stream, int a_dtype = HIF8_DTYPE_NONE);

}  // namespace hif8
