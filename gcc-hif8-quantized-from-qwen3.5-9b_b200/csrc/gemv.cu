// Split-K tensor-core GEMV for HiF8 W8A8 decode shapes (M <= 16).
//
//   y[m, n] = cast((acc[m, n] * cs[n]) * ts[m] + bias[n]),
//   acc = sum_k decode(a[m, k]) * decode(w[n, k])          (FP32 accumulate)
//
// The weight stream (N x K bytes) is the whole cost, so the kernel is built
// to keep HBM busy:
//   * each warp owns 16 weight rows and streams them with 16-byte
//     L1-bypassing loads, several 64-byte K blocks ahead in registers;
//   * a weight byte becomes BF16 with one shared-memory lookup: a 256-entry
//     table replicated per lane (entry b of lane l at byte (b << 8) | (l << 2)),
//     so every lane always hits its own bank; one PRMT builds that address
//     from the weight word and the lane offset;
//   * the decoded 16 x 16 tile feeds mma.sync m16n8k16 (BF16 in, FP32
//     accumulate) against the activation tile (8 or 16 tokens, decoded once
//     per CTA into shared memory).  Lane (g, t) takes K bytes t*16 .. t*16+15
//     of a 64-byte block, so the MMA's logical K order is a fixed
//     permutation of memory order -- applied identically to the activations;
//   * K is split over a thread-block cluster (1..8 CTAs); partial tiles are
//     reduced through distributed shared memory in a fixed order, so results
//     are deterministic and no global scratch is needed.
#include <cooperative_groups.h>

#include "linear.cuh"

namespace cg = cooperative_groups;

namespace hif8 {

constexpr int kGemvWarps = 8;
constexpr int kGemvRows = kGemvWarps * 16;  // weight rows per CTA
constexpr int kLutBytes = 256 * 256;        // lane-replicated table, 256 B per entry
constexpr int kPrefetch = 4;                // 64-byte K blocks in flight per lane

__device__ __forceinline__ uint4 ldg_stream(const uint8_t *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t lut_lookup(uint32_t lut_base, uint32_t word, uint32_t lane4, uint32_t sel) {
  const uint32_t off = __byte_perm(word, lane4, sel);
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(lut_base + off));
  return v;
}

// Decode the 4 bytes of `word` into two BF16x2 registers (bytes 0,1 and 2,3).
__device__ __forceinline__ void decode4(uint32_t lut_base, uint32_t word, uint32_t lane4, uint32_t &lo,
                                        uint32_t &hi) {
  const uint32_t e0 = lut_lookup(lut_base, word, lane4, 0x5504u);
  const uint32_t e1 = lut_lookup(lut_base, word, lane4, 0x5514u);
  const uint32_t e2 = lut_lookup(lut_base, word, lane4, 0x5524u);
  const uint32_t e3 = lut_lookup(lut_base, word, lane4, 0x5534u);
  lo = __byte_perm(e0, e1, 0x5410u);
  hi = __byte_perm(e2, e3, 0x5410u);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Activation source of the linear kernels.
constexpr int kActCodes = 0;  // HiF8 bytes
constexpr int kActBf16 = 1;   // BF16, quantised in the prologue with ts[0]
constexpr int kActF16 = 2;    // FP16, idem

// Static-quantise one FP16/BF16 value with fixed scale s and decode it back:
// the BF16 payload of decode(enc_sat(x / s)), bit-identical to running
// hif8_static_quant and then decoding its byte.
template <int ASRC>
__device__ __forceinline__ uint32_t fake_quant_bf16(uint32_t h, float s, float r, bool exact_only) {
  const float f = ASRC == kActBf16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
  float q = __fmul_rn(f, r);
  uint32_t u = __float_as_uint(q);
  const uint32_t low = u & 0x7FFFFu;
  uint32_t code;
  if (exact_only | ((low - 4u) > 0x7FFF8u) | ((u & 0x7F800000u) >= 0x7D000000u)) {
    q = __fdiv_rn(f, s);
    u = __float_as_uint(q);
    code = ((u & 0x7FFFFFFFu) > 0x7F800000u) ? 0x80u : (uint32_t)g_static_encode.v[u >> 19];
  } else {
    code = g_static_encode.v[u >> 19];
  }
  return g_decode_f32.v[code] >> 16;
}

template <int NT>
__host__ __device__ constexpr int gemv_act_stride(int kc) {
  return kc * 2 + 16;  // bytes; the 16-byte pad spreads token rows over banks
}

// The activation tile is reused for the cluster reduction after the main
// loop ([kGemvRows][8 * NT] FP32), so the region is the larger of the two.
template <int NT>
__host__ __device__ constexpr size_t gemv_smem_bytes(int kc) {
  const size_t act = (size_t)(8 * NT) * gemv_act_stride<NT>(kc);
  const size_t red = (size_t)kGemvRows * 8 * NT * sizeof(float);
  return (size_t)kLutBytes + (act > red ? act : red);
}

template <int OUT>
__device__ __forceinline__ void store_out(void *out, int64_t idx, float v) {
  if constexpr (OUT == HIF8_DTYPE_BF16) static_cast<uint16_t *>(out)[idx] = (uint16_t)f32_to_bf16_bits(v);
  else static_cast<uint16_t *>(out)[idx] = (uint16_t)f32_to_f16_bits(v);
}

__device__ __forceinline__ float load_bias(const void *bias, int dtype, int n) {
  const uint16_t h = static_cast<const uint16_t *>(bias)[n];
  return dtype == HIF8_DTYPE_BF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}

template <int NT, int OUT, int ASRC>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) gemv_hif8_kernel(const GemvArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *act = smem + kLutBytes;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ks = gridDim.y, kr = blockIdx.y;  // cluster spans the K splits
  const int k0 = kr * p.kc;
  const int act_stride = gemv_act_stride<NT>(p.kc);

  // ---- prologue: lane-replicated decode table + decoded activation tile ----
  {
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem);
    for (int i = tid; i < 256 * 32; i += blockDim.x) {
      const int b = i >> 5, l = i & 31;
      lut[b * 64 + l] = g_decode_f32.v[b] >> 16;
    }
    const int chunks_per_tok = p.kc >> 4;  // 16-byte chunks
    for (int i = tid; i < 8 * NT * chunks_per_tok; i += blockDim.x) {
      const int tok = i / chunks_per_tok, ch = i - tok * chunks_per_tok;
      uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
      if (ASRC != kActCodes && tok < p.m) {
        const float s = p.ts[0];
        const float r = __frcp_rn(s);
        const uint32_t re = __float_as_uint(r) & 0x7F800000u;
        const bool exact_only = (re == 0u) | (re == 0x7F800000u);
        const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p.a) +
                                                           (int64_t)tok * p.k + k0 + ch * 16);
        const uint4 v0 = src[0], v1 = src[1];
        const uint32_t h8[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t r8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          r8[j] = fake_quant_bf16<ASRC>(h8[j] & 0xFFFFu, s, r, exact_only) |
                  (fake_quant_bf16<ASRC>(h8[j] >> 16, s, r, exact_only) << 16);
        o0 = make_uint4(r8[0], r8[1], r8[2], r8[3]);
        o1 = make_uint4(r8[4], r8[5], r8[6], r8[7]);
      } else if (tok < p.m) {
        const uint4 v = *reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.a) + (int64_t)tok * p.k +
                                                         k0 + ch * 16);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
        uint32_t r[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t w = w4[j];
          r[2 * j] = (g_decode_f32.v[w & 0xFF] >> 16) | (g_decode_f32.v[(w >> 8) & 0xFF] & 0xFFFF0000u);
          r[2 * j + 1] = (g_decode_f32.v[(w >> 16) & 0xFF] >> 16) | (g_decode_f32.v[w >> 24] & 0xFFFF0000u);
        }
        o0 = make_uint4(r[0], r[1], r[2], r[3]);
        o1 = make_uint4(r[4], r[5], r[6], r[7]);
      }
      uint4 *dst = reinterpret_cast<uint4 *>(act + tok * act_stride + ch * 32);
      dst[0] = o0;
      dst[1] = o1;
    }
  }
  __syncthreads();

  // ---- main loop --------------------------------------------------------
  const int g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * kGemvRows + warp * 16 + g;
  const int r0 = min(row0, p.n - 1), r1 = min(row0 + 8, p.n - 1);
  const uint8_t *w0 = p.w + (int64_t)r0 * p.k + k0 + t * 16;
  const uint8_t *w1 = p.w + (int64_t)r1 * p.k + k0 + t * 16;
  const uint32_t lut_base = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t lane4 = (uint32_t)lane << 2;
  const uint32_t act_base = (uint32_t)__cvta_generic_to_shared(act) + g * act_stride + t * 32;
  const int nkb = p.kc >> 6;

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

  uint4 ring[kPrefetch][2];
#pragma unroll
  for (int s = 0; s < kPrefetch; ++s) {
    if (s < nkb) {
      ring[s][0] = ldg_stream(w0 + s * 64);
      ring[s][1] = ldg_stream(w1 + s * 64);
    }
  }

  for (int kb0 = 0; kb0 < nkb; kb0 += kPrefetch) {
#pragma unroll
    for (int s = 0; s < kPrefetch; ++s) {
      const int kb = kb0 + s;
      if (kb < nkb) {
        const uint4 x0 = ring[s][0], x1 = ring[s][1];
        if (kb + kPrefetch < nkb) {
          ring[s][0] = ldg_stream(w0 + (kb + kPrefetch) * 64);
          ring[s][1] = ldg_stream(w1 + (kb + kPrefetch) * 64);
        }
        // activation fragments of this 64-byte block: 16 BF16 per token row
        uint4 bf[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t addr = act_base + nt * 8 * act_stride + kb * 128;
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(bf[nt][0].x), "=r"(bf[nt][0].y), "=r"(bf[nt][0].z), "=r"(bf[nt][0].w)
                       : "r"(addr));
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(bf[nt][1].x), "=r"(bf[nt][1].y), "=r"(bf[nt][1].z), "=r"(bf[nt][1].w)
                       : "r"(addr + 16));
        }
        const uint32_t wa[4] = {x0.x, x0.y, x0.z, x0.w};
        const uint32_t wb[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          decode4(lut_base, wa[j], lane4, a[0], a[2]);
          decode4(lut_base, wb[j], lane4, a[1], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint4 &q = bf[nt][j >> 1];
            const uint32_t b0 = (j & 1) ? q.z : q.x;
            const uint32_t b1 = (j & 1) ? q.w : q.y;
            mma_bf16_16816(acc[nt], a, b0, b1);
          }
        }
      }
    }
  }

  // ---- reduction over the K split + epilogue -----------------------------
  const int n_a = row0, n_b = row0 + 8;
  if (ks == 1) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int m = nt * 8 + 2 * t + (q & 1);
        const int n = (q < 2) ? n_a : n_b;
        if (m < p.m && n < p.n) {
          float v = acc[nt][q] * __ldg(p.cs + n);
          v = v * __ldg(p.ts + m * p.ts_stride);
          if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
          store_out<OUT>(p.out, (int64_t)m * p.n + n, v);
        }
      }
    }
    return;
  }

  cg::cluster_group cluster = cg::this_cluster();
  float *red = reinterpret_cast<float *>(act);  // [kGemvRows][8 * NT]
  __syncthreads();                              // activation tile is dead now
  constexpr int kTok = 8 * NT;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int m = nt * 8 + 2 * t + (q & 1);
      const int rl = warp * 16 + g + ((q < 2) ? 0 : 8);
      red[rl * kTok + m] = acc[nt][q];
    }
  }
  cluster.sync();
  // CTA `kr` of the cluster reduces rows [kr * rows_per, (kr + 1) * rows_per)
  const int rows_per = kGemvRows / ks;
  const int elems = rows_per * kTok;
  for (int i = tid; i < elems; i += blockDim.x) {
    const int m = i / rows_per, rl = kr * rows_per + (i - m * rows_per);
    float v = 0.f;
    for (int r = 0; r < ks; ++r) {
      const float *remote = cluster.map_shared_rank(red, r);
      v += remote[rl * kTok + m];
    }
    const int n = blockIdx.x * kGemvRows + rl;
    if (m < p.m && n < p.n) {
      v = v * __ldg(p.cs + n);
      v = v * __ldg(p.ts + m * p.ts_stride);
      if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
      store_out<OUT>(p.out, (int64_t)m * p.n + n, v);
    }
  }
  cluster.sync();  // keep this CTA's partials alive until every reader is done
}

// Any shape, any alignment: one warp per (m, n) output, FP32 accumulation in
// a fixed per-lane order followed by a fixed shuffle tree (deterministic).
template <int OUT, int ASRC>
__global__ void __launch_bounds__(256) linear_hif8_generic(const GemvArgs p) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)p.m * p.n;
  for (int64_t o = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); o < total; o += (int64_t)gridDim.x * warps) {
    const int m = (int)(o / p.n), n = (int)(o - (int64_t)m * p.n);
    const uint8_t *w = p.w + (int64_t)n * p.k;
    float acc = 0.f;
    if constexpr (ASRC == kActCodes) {
      const uint8_t *a = static_cast<const uint8_t *>(p.a) + (int64_t)m * p.k;
      for (int k = lane; k < p.k; k += 32)
        acc = fmaf(__uint_as_float(g_decode_f32.v[a[k]]), __uint_as_float(g_decode_f32.v[w[k]]), acc);
    } else {
      const uint16_t *a = static_cast<const uint16_t *>(p.a) + (int64_t)m * p.k;
      const float s = p.ts[0];
      const float r = __frcp_rn(s);
      const uint32_t re = __float_as_uint(r) & 0x7F800000u;
      const bool exact_only = (re == 0u) | (re == 0x7F800000u);
      for (int k = lane; k < p.k; k += 32)
        acc = fmaf(__uint_as_float(fake_quant_bf16<ASRC>(a[k], s, r, exact_only) << 16),
                   __uint_as_float(g_decode_f32.v[w[k]]), acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0) {
      float v = acc * p.cs[n];
      v = v * p.ts[m * p.ts_stride];
      if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
      store_out<OUT>(p.out, o, v);
    }
  }
}

// ------------------------------------------------------------------ host --

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct GemvPlan {
  int ks = 0;   // cluster size over K (0 = fast path not applicable)
  int kc = 0;
  int nt = 1;
};

static GemvPlan plan_gemv(int64_t m, int64_t n, int64_t k) {
  GemvPlan plan;
  if (m < 1 || m > 16 || k % 64 != 0) return plan;
  plan.nt = m > 8 ? 2 : 1;
  const int64_t row_blocks = (n + kGemvRows - 1) / kGemvRows;
  const int64_t target = 2LL * num_sms();  // two co-resident CTAs per SM
  for (int ks = 1; ks <= 8; ks *= 2) {
    if (k % (64LL * ks) != 0) break;
    const int64_t kc = k / ks;
    const size_t smem = plan.nt == 2 ? gemv_smem_bytes<2>((int)kc) : gemv_smem_bytes<1>((int)kc);
    if (smem > 200 * 1024) continue;  // this split does not fit; try a finer one
    plan.ks = ks;
    plan.kc = (int)kc;
    if (row_blocks * ks >= target) break;
  }
  return plan;
}

template <int NT, int OUT, int ASRC>
static int launch_gemv(const GemvArgs &args, const GemvPlan &plan, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes<NT>(plan.kc);
  auto kernel = gemv_hif8_kernel<NT, OUT, ASRC>;
  const int st = ensure_smem_limit(reinterpret_cast<const void *>(kernel), smem);
  if (st != HIF8_OK) return st;
  cudaError_t err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((args.n + kGemvRows - 1) / kGemvRows), (unsigned)plan.ks, 1);
  cfg.blockDim = dim3(kGemvWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)plan.ks;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GemvArgs a = args;
  a.kc = plan.kc;
  err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) {
    set_last_error(err);
    return HIF8_ERR_CUDA;
  }
  return check_launch();
}

template <int OUT, int ASRC>
static int launch_generic(const GemvArgs &args, cudaStream_t stream) {
  const int64_t total = (int64_t)args.m * args.n;
  int64_t blocks = (total + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  linear_hif8_generic<OUT, ASRC><<<(unsigned)(blocks > 0 ? blocks : 1), 256, 0, stream>>>(args);
  return check_launch();
}

// y = a @ w^T for any m: the split-K tensor-core kernel on 16-token slices
// when the shape allows it, otherwise the generic kernel.
int run_linear(GemvArgs args, int output_dtype, cudaStream_t stream) {
  const bool vec_ok = aligned16(args.a) && aligned16(args.w) && args.k % 64 == 0;
  const bool bf16_out = output_dtype == HIF8_DTYPE_BF16;
  for (int m0 = 0; m0 < args.m; m0 += 16) {
    GemvArgs s = args;
    s.m = min(16, args.m - m0);
    s.a = static_cast<const uint8_t *>(args.a) + (int64_t)m0 * args.k;
    s.ts = args.ts + m0;
    s.out = static_cast<uint8_t *>(args.out) + (int64_t)m0 * args.n * 2;
    const GemvPlan plan = vec_ok ? plan_gemv(s.m, s.n, s.k) : GemvPlan{};
    int status;
    if (plan.ks == 0) {
      status = bf16_out ? launch_generic<HIF8_DTYPE_BF16, kActCodes>(s, stream)
                        : launch_generic<HIF8_DTYPE_F16, kActCodes>(s, stream);
    } else if (plan.nt == 1) {
      status = bf16_out ? launch_gemv<1, HIF8_DTYPE_BF16, kActCodes>(s, plan, stream)
                        : launch_gemv<1, HIF8_DTYPE_F16, kActCodes>(s, plan, stream);
    } else {
      status = bf16_out ? launch_gemv<2, HIF8_DTYPE_BF16, kActCodes>(s, plan, stream)
                        : launch_gemv<2, HIF8_DTYPE_F16, kActCodes>(s, plan, stream);
    }
    if (status != HIF8_OK) return status;
  }
  return HIF8_OK;
}

// Fused static quant + linear for m <= 8 rows of FP16/BF16 activations.
int run_fused_linear(const GemvArgs &args, int x_dtype, int output_dtype, cudaStream_t stream) {
  const bool bf16_out = output_dtype == HIF8_DTYPE_BF16;
  const bool bf16_in = x_dtype == HIF8_DTYPE_BF16;
  const bool vec_ok = aligned16(args.a) && aligned16(args.w) && args.k % 64 == 0 && args.m <= 8;
  const GemvPlan plan = vec_ok ? plan_gemv(args.m, args.n, args.k) : GemvPlan{};
  if (plan.ks == 0) {
    if (bf16_in)
      return bf16_out ? launch_generic<HIF8_DTYPE_BF16, kActBf16>(args, stream)
                      : launch_generic<HIF8_DTYPE_F16, kActBf16>(args, stream);
    return bf16_out ? launch_generic<HIF8_DTYPE_BF16, kActF16>(args, stream)
                    : launch_generic<HIF8_DTYPE_F16, kActF16>(args, stream);
  }
  if (bf16_in)
    return bf16_out ? launch_gemv<1, HIF8_DTYPE_BF16, kActBf16>(args, plan, stream)
                    : launch_gemv<1, HIF8_DTYPE_F16, kActBf16>(args, plan, stream);
  return bf16_out ? launch_gemv<1, HIF8_DTYPE_BF16, kActF16>(args, plan, stream)
                  : launch_gemv<1, HIF8_DTYPE_F16, kActF16>(args, plan, stream);
}

static int validate_linear(const void *a, const uint8_t *w, const float *ts, const float *cs, const void *bias,
                           int bias_dtype, int output_dtype, int64_t m, int64_t n, int64_t k, void *out) {
  if (!a || !w || !ts || !cs || !out) return HIF8_ERR_INVALID_ARGUMENT;
  if (m <= 0 || n <= 0 || k <= 0 || m > 0xFFFFFFFFLL || n > 0x7FFFFFFFLL || k > 0x7FFFFFFFLL)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (output_dtype != HIF8_DTYPE_F16 && output_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  if (bias && bias_dtype != HIF8_DTYPE_F16 && bias_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  return HIF8_OK;
}

}  // namespace hif8

using namespace hif8;

extern "C" int soft_hif8_gemv(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                              const float *channel_scale, const void *bias, int bias_dtype, int output_dtype,
                              int64_t m, int64_t n, int64_t k, void *out, void *stream) {
  int status = validate_linear(activation, weight, token_scale, channel_scale, bias, bias_dtype, output_dtype, m,
                               n, k, out);
  if (status != HIF8_OK) return status;
  if (m > 2) return HIF8_ERR_INVALID_ARGUMENT;  // reference contract: soft_hif8_gemv requires M <= 2
  GemvArgs args{activation, weight, token_scale, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                bias ? bias_dtype : HIF8_DTYPE_NONE, 1};
  return run_linear(args, output_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" size_t soft_hif8_gemm_workspace_size(int64_t m, int64_t n, int64_t k) {
  return hif8_gemm_tc_supported(m, n, k) ? hif8_gemm_tc_workspace(m, n, k) : 0;
}

extern "C" int soft_hif8_gemm(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                              const float *channel_scale, const void *bias, int bias_dtype, int output_dtype,
                              int64_t m, int64_t n, int64_t k, void *out, void *workspace,
                              size_t workspace_bytes, void *stream) {
  int status = validate_linear(activation, weight, token_scale, channel_scale, bias, bias_dtype, output_dtype, m,
                               n, k, out);
  if (status != HIF8_OK) return status;
  GemvArgs args{activation, weight, token_scale, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                bias ? bias_dtype : HIF8_DTYPE_NONE, 1};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (hif8_gemm_tc_supported(m, n, k)) {
    if (workspace_bytes < hif8_gemm_tc_workspace(m, n, k) || (!workspace && hif8_gemm_tc_workspace(m, n, k)))
      return HIF8_ERR_WORKSPACE;
    return hif8_gemm_tc(args, output_dtype, workspace, workspace_bytes, s);
  }
  return run_linear(args, output_dtype, s);
}

extern "C" int soft_hif8_static_fused_gemm(const void *x, int x_dtype, const uint8_t *weight,
                                          const float *fixed_scale, const float *channel_scale, const void *bias,
                                          int bias_dtype, int output_dtype, int64_t m, int64_t n, int64_t k,
                                          void *out, void *stream) {
  int status = validate_linear(x, weight, fixed_scale, channel_scale, bias, bias_dtype, output_dtype, m, n, k, out);
  if (status != HIF8_OK) return status;
  if (m > 4) return HIF8_ERR_INVALID_ARGUMENT;  // reference contract: M <= 4
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  GemvArgs args{x, weight, fixed_scale, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                bias ? bias_dtype : HIF8_DTYPE_NONE, 0};
  return run_fused_linear(args, x_dtype, output_dtype, static_cast<cudaStream_t>(stream));
}
