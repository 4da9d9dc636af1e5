// Persistent split-K tensor-core GEMV for HiF8 W8A8 decode shapes (M <= 16).
//
//   y[m, n] = cast((acc[m, n] * cs[n]) * ts[m] + bias[n]),
//   acc = sum_k decode(a[m, k]) * decode(w[n, k])          (FP32 accumulate)
//
// The weight stream (N x K bytes) is the whole cost; the kernel is shaped to
// keep HBM busy from every SM for the whole launch:
//   * one persistent CTA of 16 warps per SM (grid = SMs, rounded to whole
//     clusters), so the 64 KB lane-replicated decode table and the activation
//     tile are built once per SM;
//   * K is split over a thread-block cluster of S CTAs (rank = K slice); each
//     cluster walks row blocks ("items") round-robin, so every CTA keeps one
//     K slice of the activation decoded in shared memory for the whole launch;
//   * inside a CTA the 16 warps split the item as WR row groups x WK K parts;
//     every warp always owns exactly two 128-byte K blocks per item, so its
//     2-deep register ring of 32-byte weight loads (one 128-byte row segment
//     per four lanes: a load instruction of the warp moves 1 KB) is indexed
//     at compile time and runs straight across item boundaries (the next
//     item's blocks are in flight while the current one is reduced);
//   * a weight byte becomes BF16 with one shared-memory lookup: entry b of
//     lane l sits at byte (b << 8) | (l << 2), so a lane always hits its own
//     bank, and one PRMT builds the address from the weight word;
//   * decoded 16 x 16 weight tiles feed mma.sync m16n8k16 (BF16, FP32
//     accumulate) against the activation fragments.  Lane (g, t) takes bytes
//     t*32 .. t*32+31 of a 128-byte block, so the MMA's K order is a fixed
//     permutation of memory order, applied identically to the activations
//     (stored in that order, 16-byte chunks rotated so the fragment loads are
//     free of bank conflicts; rows of padding tokens are not loaded);
//   * partial sums are reduced in a fixed order: the warps of an item after
//     every item (or of all items at the end, for M <= 4), then the cluster
//     ranks: every rank stores its partials into the owning rank's shared
//     memory (distributed shared memory) as they are produced, and each rank
//     sums the slots of its share once, at the end -- deterministic, no
//     global scratch.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/hif8_b200_model.h"
#include "linear.cuh"

namespace cg = cooperative_groups;

namespace hif8 {

constexpr int kWarps = 16;                  // warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kLutBytes = 256 * 256;        // lane-replicated table, 256 B per entry
constexpr int kBlk = 128;                   // K bytes of one ring stage (32 per lane of a row)
constexpr int kRing = 2;                    // K blocks per warp per item (= ring depth)
constexpr int kWarpK = kRing * kBlk;        // K per warp per item
constexpr int kRedStride = 20;              // floats per token row of a warp partial (bank-conflict-free)

// Activation source of the linear kernels.
constexpr int kActCodes = 0;  // HiF8 bytes
constexpr int kActBf16 = 1;   // BF16, quantised in the prologue with ts[0]
constexpr int kActF16 = 2;    // FP16, idem
// BF16 produced in the prologue by a fused glue step (p.glue), then quantised
constexpr int kActSiluMul = 3;
constexpr int kActGateMul = 4;
constexpr int kActRmsNorm = 5;

template <int ASRC>
__host__ __device__ constexpr bool act_is_glue() {
  return ASRC == kActSiluMul || ASRC == kActGateMul || ASRC == kActRmsNorm;
}

// BF16 bits of the glue step for one element: x (and y: up / gate /
// residual, w: norm weight) are BF16 bits; the arithmetic and its roundings
// are those of the separate model kernels (silu_mul, gate_mul, rmsnorm).
template <int ASRC>
__device__ __forceinline__ uint32_t glue_value(uint32_t x, uint32_t y, uint32_t w, float inv, bool has_y,
                                               bool one_plus) {
  if constexpr (ASRC == kActSiluMul) {
    return f32_to_bf16_bits(glue_silu(bf16_bits_to_f32(x)) * bf16_bits_to_f32(y));
  } else if constexpr (ASRC == kActGateMul) {
    return f32_to_bf16_bits(bf16_bits_to_f32(x) * glue_sigmoid(bf16_bits_to_f32(y)));
  } else {
    float v = bf16_bits_to_f32(x);
    if (has_y) v = bf16_bits_to_f32(f32_to_bf16_bits(v + bf16_bits_to_f32(y)));  // BF16 residual stream
    float ww = bf16_bits_to_f32(w);
    if (one_plus) ww += 1.f;
    return f32_to_bf16_bits(v * inv * ww);
  }
}

struct U32x8 {
  uint32_t v[8];
};

// 32 bytes per lane (a 256-bit load; p 32-byte aligned), streamed past L1.
__device__ __forceinline__ U32x8 ldg_stream32(const uint8_t *p) {
  U32x8 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
                 "=r"(r.v[6]), "=r"(r.v[7])
               : "l"(p));
  return r;
}

// Byte offset, inside one token row of the activation tile, of the 8 BF16
// values at K index kk (kk % 8 == 0) of the CTA's slice.  Block b of 128 K
// holds lane quarter tq's 32 values at tq*64; their four 16-byte chunks are
// rotated by 2*(tq>>1) so that lanes t = 0..3 reading chunk c hit four
// different 16-byte bank groups.
__device__ __forceinline__ int act_offset(int kk) {
  const int b = kk >> 7, w = kk & 127, tq = w >> 5, c = (w >> 3) & 3;
  return b * 256 + tq * 64 + (((c + 2 * (tq >> 1)) & 3) << 4);
}

__device__ __forceinline__ uint32_t lut_lookup(const uint8_t *lut, uint32_t word, uint32_t lane4, uint32_t sel) {
  return *reinterpret_cast<const uint32_t *>(lut + __byte_perm(word, lane4, sel));
}

// Decode the 4 bytes of `word` into two BF16x2 registers (bytes 0,1 and 2,3).
__device__ __forceinline__ void decode4(const uint8_t *lut, uint32_t word, uint32_t lane4, uint32_t &lo,
                                        uint32_t &hi) {
  const uint32_t e0 = lut_lookup(lut, word, lane4, 0x5504u);
  const uint32_t e1 = lut_lookup(lut, word, lane4, 0x5514u);
  const uint32_t e2 = lut_lookup(lut, word, lane4, 0x5524u);
  const uint32_t e3 = lut_lookup(lut, word, lane4, 0x5534u);
  lo = __byte_perm(e0, e1, 0x5410u);
  hi = __byte_perm(e2, e3, 0x5410u);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

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

template <int OUT>
__device__ __forceinline__ void store_out(void *out, int64_t idx, float v) {
  if constexpr (OUT == HIF8_DTYPE_BF16) static_cast<uint16_t *>(out)[idx] = (uint16_t)f32_to_bf16_bits(v);
  else if constexpr (OUT == HIF8_DTYPE_F32) static_cast<float *>(out)[idx] = v;  // TP partial products
  else static_cast<uint16_t *>(out)[idx] = (uint16_t)f32_to_f16_bits(v);
}

__device__ __forceinline__ float load_bias(const void *bias, int dtype, int n) {
  const uint16_t h = static_cast<const uint16_t *>(bias)[n];
  return dtype == HIF8_DTYPE_BF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
}

// Launch geometry of one call (host-computed).
struct GemvPlan {
  int s = 0;        // cluster size = number of K slices (0: not applicable)
  int kc = 0;       // K slice per CTA
  int wk = 0;       // warps splitting an item's K slice (kc = wk * kWarpK)
  int wr = 0;       // row groups of 16 per item (wr * wk == kWarps)
  int nt = 1;       // 8-token MMA tiles (1: M <= 8, 2: M <= 16)
  int clusters = 0;
  int max_items = 0;  // row blocks per cluster (upper bound)
  // > 0 (m <= 4): every warp keeps its partial sums of up to this many items
  // in shared memory and the items are reduced once, after the last one,
  // instead of behind a CTA barrier after every item
  int defer_items = 0;
};

// Shared memory of the deferred per-warp partials: [item][warp][m][16 rows].
__host__ __device__ constexpr size_t defer_bytes(int m, int items) {
  return (size_t)items * kWarps * m * 16 * sizeof(float);
}

// kc * 2 is a multiple of 512, so consecutive token rows start 16 bytes
// (one bank group) apart modulo 128.
__host__ __device__ constexpr int act_stride_bytes(int kc) { return kc * 2 + 16; }

// Floats of the split-K receive buffer: S slots of ceil(total / S) partials,
// total <= max_items * rows * tokens, so S - 1 floats of rounding at most.
__host__ __device__ constexpr size_t gemv_part_floats(int nt, int wr, int max_items) {
  return max_items > 0 ? (size_t)max_items * (16 * wr) * 8 * nt + 8 : 0;
}

// shared memory: table | activation tile | warp partials x2 | the split-K
// receive buffer (partials of this rank's share of the cluster's outputs,
// pushed by every rank; reduced once, at the end)
__host__ __device__ constexpr size_t gemv_smem_bytes(int nt, int kc, int wr, int max_items) {
  return (size_t)kLutBytes + (size_t)(8 * nt) * act_stride_bytes(kc) +
         2 * (size_t)kWarps * (8 * nt) * kRedStride * sizeof(float) + gemv_part_floats(nt, wr, max_items) * sizeof(float);
}

template <int NT, int OUT, int ASRC>
__global__ void __launch_bounds__(kThreads, 1) gemv_hif8_kernel(const GemvArgs p, const GemvPlan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kTok = 8 * NT;
  constexpr bool kGlue = act_is_glue<ASRC>();
  constexpr int QSRC = kGlue ? kActBf16 : ASRC;  // element type the quantiser sees
  __shared__ float norm_part[kWarps][8], norm_inv[8];  // kActRmsNorm: per-token sums / inverse RMS
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = plan.s, kc = plan.kc, WK = plan.wk, WR = plan.wr;
  const int rank = (int)(blockIdx.x % S), cluster_id = (int)(blockIdx.x / S);
  const int k0 = rank * kc;
  const int act_stride = act_stride_bytes(kc);
  uint8_t *act = smem + kLutBytes;
  float *red = reinterpret_cast<float *>(act + (size_t)kTok * act_stride);  // [2][kWarps][kTok][kRedStride]
  float *part = red + 2 * kWarps * kRedStride * kTok;                       // [S][share] received partials
  float *wpd = part + gemv_part_floats(NT, WR, plan.max_items);              // deferred: [item][warp][m][16]
  // split-K ranks store into each other's shared memory from the first item
  // on: every CTA of the cluster must have started (arrive here, wait before
  // the first store)
  if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // ---- work assignment -----------------------------------------------------
  const int g = lane >> 2, t = lane & 3;
  const int wr = warp / WK, wk = warp - wr * WK;  // row group / K part of this warp
  const int rows_per_item = 16 * WR;
  const int n_items = (p.n + rows_per_item - 1) / rows_per_item;
  const int my_items = n_items > cluster_id ? (n_items - cluster_id + plan.clusters - 1) / plan.clusters : 0;
  const int kw0 = k0 + wk * kWarpK;  // this warp's K offset inside every item

  auto weight_ptrs = [&](int item, const uint8_t *&w0, const uint8_t *&w1) {
    const int row = (cluster_id + item * plan.clusters) * rows_per_item + wr * 16 + g;
    const int r0 = min(row, p.n - 1), r1 = min(row + 8, p.n - 1);
    w0 = p.w + (int64_t)r0 * p.k + kw0 + t * 32;
    w1 = p.w + (int64_t)r1 * p.k + kw0 + t * 32;
  };

  U32x8 ring[kRing][2];

  // ---- prologue: lane-replicated decode table + this rank's activation slice
  {
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem);
    // the fused quantiser's tables, staged in the reduction buffer (idle
    // until the first item is reduced): the fake-quant table (decoded BF16 of
    // the static code per magnitude index, 8 KB) and the magnitude encode
    // table of the exact path (4 KB)
    uint16_t *fq = reinterpret_cast<uint16_t *>(red);
    uint8_t *mag = reinterpret_cast<uint8_t *>(red) + 8192;
    // Module constants only before the dependency wait: the tables are built
    // while the previous kernel of the stream completes.  warp w owns table
    // entries 16 w .. 16 w + 15 (one load per lane).
    {
      const uint32_t mine = g_decode_f32.v[warp * 16 + (lane & 15)] >> 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) lut[(warp * 16 + j) * 64 + lane] = __shfl_sync(0xFFFFFFFFu, mine, j);
      static_assert(kThreads == 512, "one fake-quant table piece per thread");
      if (ASRC != kActCodes) {
        reinterpret_cast<uint4 *>(fq)[tid] = reinterpret_cast<const uint4 *>(g_fake_quant_bf16.v)[tid];
        if (tid < 256) reinterpret_cast<uint4 *>(mag)[tid] = reinterpret_cast<const uint4 *>(g_static_encode_mag.v)[tid];
      }
    }
    // Every other global read of the prologue may depend on the previous
    // kernel of the stream (its activations, or weights it has just
    // written), so it follows the dependency wait.  The activation loads and
    // this warp's first item of weights are all issued before any of them is
    // used, so their latencies overlap instead of adding up.
    pdl_wait();
    float ts0 = 1.f;  // the fused quantiser's fixed scale
    if (ASRC != kActCodes) ts0 = p.ts[0];
    const int chunks_per_tok = kc >> 4;  // 16 K values per chunk
    // only the real tokens' rows: fragment rows of padding tokens (>= m) are
    // never loaded, so their tile rows are never written either
    const int real = (p.m < kTok ? p.m : kTok) * chunks_per_tok;
    // kPro chunks per thread and round: a round's global loads are issued
    // before its arithmetic (the first round's before the table stores)
    constexpr int kPro = kGlue ? 2 : 4;
    const int64_t a_stride = ASRC == kActSiluMul ? 2 * (int64_t)p.k : (int64_t)p.k;
    uint4 raw[kPro][2], aux[kPro][2], nw[kPro][2];
    auto load_round = [&](int base) {
#pragma unroll
      for (int u = 0; u < kPro; ++u) {
        const int i = base + u * kThreads + tid;
        raw[u][0] = raw[u][1] = aux[u][0] = aux[u][1] = nw[u][0] = nw[u][1] = make_uint4(0, 0, 0, 0);
        if (i < real) {
          const int tok = i / chunks_per_tok, ch = i - tok * chunks_per_tok;
          if (ASRC != kActCodes) {
            const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p.a) +
                                                               (int64_t)tok * a_stride + k0 + ch * 16);
            raw[u][0] = src[0];
            raw[u][1] = src[1];
            if constexpr (kGlue) {
              const uint4 *asrc =
                  ASRC == kActSiluMul ? src + p.k / 8  // up half of the gate_up row
                  : p.glue.aux ? reinterpret_cast<const uint4 *>(p.glue.aux + (int64_t)tok * p.k + k0 + ch * 16)
                               : nullptr;
              if (asrc) {
                aux[u][0] = asrc[0];
                aux[u][1] = asrc[1];
              }
              if (ASRC == kActRmsNorm) {
                const uint4 *wsrc = reinterpret_cast<const uint4 *>(p.glue.norm_w + k0 + ch * 16);
                nw[u][0] = wsrc[0];
                nw[u][1] = wsrc[1];
              }
            }
          } else {
            raw[u][0] = *reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.a) + (int64_t)tok * p.k +
                                                         k0 + ch * 16);
          }
        }
      }
    };
    load_round(0);

    if constexpr (ASRC == kActRmsNorm) {
      // inverse RMS of every token's full row (x + residual), identical in
      // every CTA; CTA 0 also writes the new BF16 residual stream
      const uint16_t *xa = static_cast<const uint16_t *>(p.a);
      const uint16_t *res = p.glue.aux;
      const bool write_res = res && p.glue.residual_out && blockIdx.x == 0;
      const int mt0 = p.m < kTok ? p.m : kTok;
      for (int tok = 0; tok < mt0; ++tok) {
        float ss = 0.f;
        for (int c = tid * 8; c < p.k; c += kThreads * 8) {
          const uint4 xv = *reinterpret_cast<const uint4 *>(xa + (int64_t)tok * p.k + c);
          uint4 rv = make_uint4(0, 0, 0, 0);
          if (res) rv = *reinterpret_cast<const uint4 *>(res + (int64_t)tok * p.k + c);
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, rw[4] = {rv.x, rv.y, rv.z, rv.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float lo = bf16_bits_to_f32(xw[i] & 0xFFFFu), hi = bf16_bits_to_f32(xw[i] >> 16);
            if (res) {
              lo = bf16_bits_to_f32(f32_to_bf16_bits(lo + bf16_bits_to_f32(rw[i] & 0xFFFFu)));
              hi = bf16_bits_to_f32(f32_to_bf16_bits(hi + bf16_bits_to_f32(rw[i] >> 16)));
            }
            o[i] = f32_to_bf16_bits(lo) | (f32_to_bf16_bits(hi) << 16);
            ss += lo * lo + hi * hi;
          }
          if (write_res)
            *reinterpret_cast<uint4 *>(p.glue.residual_out + (int64_t)tok * p.k + c) = make_uint4(o[0], o[1], o[2], o[3]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        if (lane == 0) norm_part[warp][tok] = ss;
      }
      __syncthreads();
      if (tid < mt0) {
        float tsum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tsum += norm_part[w][tid];
        norm_inv[tid] = rsqrtf(tsum / (float)p.k + p.glue.eps);
      }
    }
    __syncthreads();
    const uint32_t lane4 = (uint32_t)lane << 2;
    float r = 1.f;
    double r64 = 1.0;
    bool exact_only = false;
    if (ASRC != kActCodes) {
      r = __frcp_rn(ts0);
      r64 = __drcp_rn((double)ts0);
      const uint32_t re = __float_as_uint(r) & 0x7F800000u;
      // the exact FP64 path for every element: zero, negative and non-finite
      // scales, extreme reciprocals, and scales outside [2^-60, 2^60]
      exact_only = (re == 0u) | (re == 0x7F800000u) | !(ts0 > 0.f) | !scale_edge_ok(ts0);
    }
    const float s_half = 0.5f * ts0;
    for (int base = 0; base < real; base += kPro * kThreads) {
      if (base > 0) load_round(base);
#pragma unroll
      for (int u = 0; u < kPro; ++u) {
        const int i = base + u * kThreads + tid;
        if (i >= real) break;
        const int tok = i / chunks_per_tok, ch = i - tok * chunks_per_tok;
        uint4 o0, o1;
        {
          if (ASRC != kActCodes) {
            uint32_t h8[8] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w,
                              raw[u][1].x, raw[u][1].y, raw[u][1].z, raw[u][1].w};
            if constexpr (kGlue) {
              const uint32_t y8[8] = {aux[u][0].x, aux[u][0].y, aux[u][0].z, aux[u][0].w,
                                      aux[u][1].x, aux[u][1].y, aux[u][1].z, aux[u][1].w};
              const uint32_t w8[8] = {nw[u][0].x, nw[u][0].y, nw[u][0].z, nw[u][0].w,
                                      nw[u][1].x, nw[u][1].y, nw[u][1].z, nw[u][1].w};
              const float inv = ASRC == kActRmsNorm ? norm_inv[tok] : 1.f;
              const bool has_y = ASRC == kActSiluMul || p.glue.aux != nullptr;
              const bool one_plus = p.glue.one_plus != 0;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                h8[j] = glue_value<ASRC>(h8[j] & 0xFFFFu, y8[j] & 0xFFFFu, w8[j] & 0xFFFFu, inv, has_y, one_plus) |
                        (glue_value<ASRC>(h8[j] >> 16, y8[j] >> 16, w8[j] >> 16, inv, has_y, one_plus) << 16);
            }
            // decode(static code) of the 16 values, bit-identical to
            // hif8_static_quant and a decode of its bytes: the fake-quant
            // entry of each correctly rounded quotient, or the exact FP64
            // path (a huge or non-finite product, or a scale that needs it)
            uint32_t r8[8];
            if (exact_only || !fake_quant16<QSRC>(h8, ts0, r, s_half, fq, r8)) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                r8[j] = lut[static_code_exact(half_bits_to_f32<QSRC>(h8[j] & 0xFFFFu), r64, mag) * 64 + lane] |
                        (lut[static_code_exact(half_bits_to_f32<QSRC>(h8[j] >> 16), r64, mag) * 64 + lane] << 16);
            }
            o0 = make_uint4(r8[0], r8[1], r8[2], r8[3]);
            o1 = make_uint4(r8[4], r8[5], r8[6], r8[7]);
          } else {
            const uint32_t w4[4] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w};
            uint32_t rr[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) decode4(smem, w4[j], lane4, rr[2 * j], rr[2 * j + 1]);
            o0 = make_uint4(rr[0], rr[1], rr[2], rr[3]);
            o1 = make_uint4(rr[4], rr[5], rr[6], rr[7]);
          }
        }
        uint8_t *row = act + tok * act_stride;
        *reinterpret_cast<uint4 *>(row + act_offset(ch * 16)) = o0;
        *reinterpret_cast<uint4 *>(row + act_offset(ch * 16 + 8)) = o1;
      }
    }
    // The first item's weights after this thread's activation work: issued
    // before it, the burst of HBM reads from every SM (~10 MB) queued ahead
    // of the activation reads and delayed them by microseconds; issued as
    // soon as those reads had returned it was slower again (configs[1]
    // sweep: 328 us before, 318 us after, 328 us at the earlier point).
    if (my_items > 0) {
      const uint8_t *w0, *w1;
      weight_ptrs(0, w0, w1);
#pragma unroll
      for (int st = 0; st < kRing; ++st) {
        ring[st][0] = ldg_stream32(w0 + st * kBlk);
        ring[st][1] = ldg_stream32(w1 + st * kBlk);
      }
    }
  }
  __syncthreads();

  const int mt = p.m < kTok ? p.m : kTok;  // real tokens of the tile
  const uint8_t *lut = smem;
  const uint32_t lane4 = (uint32_t)lane << 2;
  // this lane's 64 bytes of every 128-K block: token row g (+ 8 for the
  // second tile); rows of padding tokens (>= m) are never loaded
  const uint8_t *act_lane = act + g * act_stride + (wk * kWarpK / kBlk) * 256 + t * 64;
  const int rot = 2 * (t >> 1);
  bool tok_real[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) tok_real[nt] = nt * 8 + g < p.m;

  cg::cluster_group cluster = cg::this_cluster();
  // Cross-rank reduction by push: the (item, token, row) outputs of the
  // cluster are split into S contiguous shares; rank r owns share r, and every
  // rank stores its partial of an output into slot [its rank] of the owner's
  // receive buffer as soon as the item is reduced over its warps, so the
  // transfers overlap the streaming of the next items and the end phase reads
  // only local shared memory.
  const int per_item = rows_per_item * mt;
  const int share = S > 1 ? (my_items * per_item + S - 1) / S : 0;
  auto push = [&](int idx, float v) {
    const int owner = idx / share;
    cluster.map_shared_rank(part, owner)[rank * share + (idx - owner * share)] = v;
  };
  if (S > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  for (int item = 0; item < my_items; ++item) {
    const uint8_t *n0 = nullptr, *n1 = nullptr;
    const bool has_next = item + 1 < my_items;
    if (has_next) weight_ptrs(item + 1, n0, n1);

    float acc[2][NT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[h][nt][0] = acc[h][nt][1] = acc[h][nt][2] = acc[h][nt][3] = 0.f;

#pragma unroll
    for (int s = 0; s < kRing; ++s) {
      const U32x8 x0 = ring[s][0], x1 = ring[s][1];
      if (has_next) {  // the next item's block s goes into the freed slot
        ring[s][0] = ldg_stream32(n0 + s * kBlk);
        ring[s][1] = ldg_stream32(n1 + s * kBlk);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16-byte chunk c: K t*32 + 8c .. +7 of the block
        uint4 bf[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          bf[nt] = make_uint4(0, 0, 0, 0);
          if (tok_real[nt])
            bf[nt] = *reinterpret_cast<const uint4 *>(act_lane + nt * 8 * act_stride + s * 256 +
                                                      (((c + rot) & 3) << 4));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = 2 * c + h;
          uint32_t a[4];
          decode4(lut, x0.v[j], lane4, a[0], a[2]);
          decode4(lut, x1.v[j], lane4, a[1], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_bf16_16816(acc[h][nt], a, h ? bf[nt].z : bf[nt].x, h ? bf[nt].w : bf[nt].y);
        }
      }
    }

    if (plan.defer_items) {  // keep this warp's partials of the item; no barrier
      float *dst = wpd + ((size_t)item * kWarps + warp) * mt * 16;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int m = 2 * t + (q & 1);
        if (m < mt) dst[m * 16 + g + ((q < 2) ? 0 : 8)] = acc[0][0][q] + acc[1][0][q];
      }
      continue;
    }
    // ---- reduce the item: warps (fixed order), then cluster ranks ---------
    // Partials are token-major ([token][row]) so the summing threads walk the
    // output rows of one token consecutively: the global stores coalesce.
    const int buf = item & 1;
    float *wred = red + ((size_t)buf * kWarps + warp) * kTok * kRedStride;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int m = nt * 8 + 2 * t + (q & 1);
        const int rl = g + ((q < 2) ? 0 : 8);
        wred[m * kRedStride + rl] = acc[0][nt][q] + acc[1][nt][q];
      }
    }
    __syncthreads();
    const int row_base = (cluster_id + item * plan.clusters) * rows_per_item;
    for (int e = tid; e < rows_per_item * mt; e += kThreads) {
      const int m = e / rows_per_item, rl = e - m * rows_per_item;  // token, row within the item
      const int grp = rl >> 4, r16 = rl & 15;
      const float *src = red + (((size_t)buf * kWarps + grp * WK) * kTok + m) * kRedStride + r16;
      float v = 0.f;
      for (int w = 0; w < WK; ++w) v += src[(size_t)w * kTok * kRedStride];
      if (S == 1) {
        const int n = row_base + rl;
        if (n < p.n) {
          v = v * __ldg(p.cs + n);
          v = v * __ldg(p.ts + m * p.ts_stride);
          if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
          store_out<OUT>(p.out, (int64_t)m * p.n + n, v);
        }
      } else {
        push(item * per_item + e, v);
      }
    }
  }
  if (plan.defer_items) {
    // every item at once: the WK warps of a row group summed in warp order
    __syncthreads();
    for (int e = tid; e < my_items * per_item; e += kThreads) {
      const int item = e / per_item, rem = e - item * per_item;
      const int m = rem / rows_per_item, rl = rem - m * rows_per_item;
      const int grp = rl >> 4, r16 = rl & 15;
      const float *src = wpd + ((size_t)item * kWarps + grp * WK) * mt * 16 + m * 16 + r16;
      float v = 0.f;
      for (int w = 0; w < WK; ++w) v += src[(size_t)w * mt * 16];
      if (S == 1) {
        const int n = (cluster_id + item * plan.clusters) * rows_per_item + rl;
        if (n < p.n) {
          v = v * __ldg(p.cs + n);
          v = v * __ldg(p.ts + m * p.ts_stride);
          if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
          store_out<OUT>(p.out, (int64_t)m * p.n + n, v);
        }
      } else {
        push(e, v);
      }
    }
  }
  if (S == 1) return;

  // ---- cross-rank reduction, once: the barrier makes every rank's pushed
  // partials visible; rank r sums its share's S slots in rank order
  // (deterministic) and consecutive threads store consecutive rows.  Nothing
  // reads another CTA's shared memory after the barrier, so no CTA waits for
  // its peers before leaving.
  cluster.sync();
  const int e_begin = rank * share;
  const int e_end = min(my_items * per_item, e_begin + share);
  for (int e = e_begin + tid; e < e_end; e += kThreads) {
    const int item = e / per_item, rem = e - item * per_item;
    const int m = rem / rows_per_item, rl = rem - m * rows_per_item;
    float v = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < S) v += part[r * share + (e - e_begin)];
    const int n = (cluster_id + item * plan.clusters) * rows_per_item + rl;
    if (n < p.n) {
      v = v * __ldg(p.cs + n);
      v = v * __ldg(p.ts + m * p.ts_stride);
      if (p.bias) v += load_bias(p.bias, p.bias_dtype, n);
      store_out<OUT>(p.out, (int64_t)m * p.n + n, v);
    }
  }
}

// Any shape, any alignment: one warp per (m, n) output, FP32 accumulation in
// a fixed per-lane order followed by a fixed shuffle tree (deterministic).
template <int OUT, int ASRC>
__global__ void __launch_bounds__(256) linear_hif8_generic(const GemvArgs p) {
  pdl_wait();
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
static bool aligned32(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

constexpr size_t kMaxSmem = 227 * 1024;

// Dynamic shared memory a kernel may request: the per-block limit less its
// static shared memory (cached per kernel).
static size_t dyn_smem_cap(const void *kernel) {
  static std::mutex mu;
  static std::vector<std::pair<const void *, size_t>> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto &e : cache)
    if (e.first == kernel) return e.second;
  cudaFuncAttributes attr{};
  size_t cap = kMaxSmem;
  if (cudaFuncGetAttributes(&attr, kernel) == cudaSuccess) cap = kMaxSmem - std::min(kMaxSmem, attr.sharedSizeBytes);
  else cudaGetLastError();
  cache.push_back({kernel, cap});
  return cap;
}

// Clusters of `s` CTAs of `kernel` that can be resident at once (cached per
// device, kernel, cluster size and shared-memory size).
static int max_active_clusters(const void *kernel, int s, size_t smem_request) {
  const size_t smem = std::min(smem_request, dyn_smem_cap(kernel));
  struct Entry {
    const void *kernel;
    int device, s;
    size_t smem;
    int clusters;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry &e : cache)
      if (e.kernel == kernel && e.device == dev && e.s == s && e.smem == smem) return e.clusters;
  }
  const int sms = num_sms();
  int clusters = sms / s;
  if (ensure_smem_limit(kernel, smem) == HIF8_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(s * (sms / s)), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)s;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess && n > 0) clusters = n < clusters ? n : clusters;
    else cudaGetLastError();
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({kernel, dev, s, smem, clusters});
  return clusters;
}

// Pick the K split S (cluster size) and the warp arrangement that balance the
// rounds of row blocks over the co-resident persistent clusters best.
static GemvPlan plan_gemv(int64_t m, int64_t n, int64_t k, const void *kernel) {
  GemvPlan best;
  if (m < 1 || m > 16 || n < 1 || k % kWarpK != 0) return best;
  const int nt = m > 8 ? 2 : 1;
  const int sms = num_sms();
  double best_eff = -1.0;
  for (int s = 1; s <= 8; ++s) {
    if (k % ((int64_t)s * kWarpK) != 0) continue;
    const int64_t kc = k / s;
    if (kc % kWarpK != 0) continue;
    const int64_t wk = kc / kWarpK;
    if (wk > kWarps || kWarps % wk != 0) continue;
    const int wr = (int)(kWarps / wk);
    const int64_t items = (n + 16 * wr - 1) / (16 * wr);
    // shared memory is sized for the worst case of sms / s clusters
    const int64_t rounds_max = (items + (sms / s) - 1) / (sms / s);
    const size_t cap = dyn_smem_cap(kernel);
    const size_t smem = gemv_smem_bytes(nt, (int)kc, wr, s > 1 ? (int)std::max<int64_t>(rounds_max, items) : 0);
    if (gemv_smem_bytes(nt, (int)kc, wr, 0) > cap) continue;
    const int clusters = max_active_clusters(kernel, s, std::min(smem, cap));
    if (clusters < 1) continue;
    const int64_t rounds = (items + clusters - 1) / clusters;
    if (gemv_smem_bytes(nt, (int)kc, wr, s > 1 ? (int)rounds : 0) > cap) continue;
    // fraction of the machine's CTA-rounds doing useful work
    const double eff = (double)items / (double)(rounds * clusters) * (double)(clusters * s) / (double)sms;
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best.s = s;
      best.kc = (int)kc;
      best.wk = (int)wk;
      best.wr = wr;
      best.nt = nt;
      best.clusters = clusters;
      best.max_items = s > 1 ? (int)rounds : 0;
      // deferred reduction for up to 4 tokens when its partials fit
      const size_t base = gemv_smem_bytes(nt, (int)kc, wr, s > 1 ? (int)rounds : 0);
      best.defer_items = (nt == 1 && m <= 4 && base + defer_bytes((int)m, (int)rounds) <= cap) ? (int)rounds : 0;
    }
  }
  return best;
}

// plan_gemv memoised per (device, kernel, m, n, k): the plan is a pure
// function of those, and the search costs microseconds of host time per call
// (an eager decode step makes dozens of calls).
static GemvPlan plan_gemv_cached(int64_t m, int64_t n, int64_t k, const void *kernel) {
  struct Entry {
    const void *kernel;
    int device;
    int64_t m, n, k;
    GemvPlan plan;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry &e : cache)
      if (e.kernel == kernel && e.device == dev && e.m == m && e.n == n && e.k == k) return e.plan;
  }
  const GemvPlan plan = plan_gemv(m, n, k, kernel);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() < 4096) cache.push_back({kernel, dev, m, n, k, plan});
  return plan;
}

template <int NT, int OUT, int ASRC>
static const void *gemv_kernel_ptr() {
  return reinterpret_cast<const void *>(gemv_hif8_kernel<NT, OUT, ASRC>);
}

template <int NT, int OUT, int ASRC>
static int launch_gemv(const GemvArgs &args, const GemvPlan &plan, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(NT, plan.kc, plan.wr, plan.max_items) + defer_bytes(args.m, plan.defer_items);
  auto kernel = gemv_hif8_kernel<NT, OUT, ASRC>;
  const int st = ensure_smem_limit(reinterpret_cast<const void *>(kernel), smem);
  if (st != HIF8_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(plan.clusters * plan.s), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)plan.s;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args, plan);
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
  return launch_pdl(linear_hif8_generic<OUT, ASRC>, dim3((unsigned)(blocks > 0 ? blocks : 1)), dim3(256), 0, stream,
                    args);
}

// y = a @ w^T for any m: the persistent split-K kernel on 16-token slices
// when the shape allows it, otherwise the generic kernel.
template <int OUT>
static int run_linear_out(GemvArgs args, cudaStream_t stream) {
  // 16-byte activation loads, 32-byte weight loads (k % 256 == 0 keeps every
  // row segment aligned)
  const bool vec_ok = aligned16(args.a) && aligned32(args.w) && args.k % 64 == 0;
  constexpr int64_t out_bytes = OUT == HIF8_DTYPE_F32 ? 4 : 2;
  for (int m0 = 0; m0 < args.m; m0 += 16) {
    GemvArgs s = args;
    s.m = min(16, args.m - m0);
    s.a = static_cast<const uint8_t *>(args.a) + (int64_t)m0 * args.k;
    s.ts = args.ts + m0;
    s.out = static_cast<uint8_t *>(args.out) + (int64_t)m0 * args.n * out_bytes;
    const void *kptr = s.m > 8 ? gemv_kernel_ptr<2, OUT, kActCodes>() : gemv_kernel_ptr<1, OUT, kActCodes>();
    const GemvPlan plan = vec_ok ? plan_gemv_cached(s.m, s.n, s.k, kptr) : GemvPlan{};
    int status;
    if (plan.s == 0) status = launch_generic<OUT, kActCodes>(s, stream);
    else if (plan.nt == 1) status = launch_gemv<1, OUT, kActCodes>(s, plan, stream);
    else status = launch_gemv<2, OUT, kActCodes>(s, plan, stream);
    if (status != HIF8_OK) return status;
  }
  return HIF8_OK;
}

int run_linear(GemvArgs args, int output_dtype, cudaStream_t stream) {
  switch (output_dtype) {
    case HIF8_DTYPE_BF16: return run_linear_out<HIF8_DTYPE_BF16>(args, stream);
    case HIF8_DTYPE_F16: return run_linear_out<HIF8_DTYPE_F16>(args, stream);
    case HIF8_DTYPE_F32: return run_linear_out<HIF8_DTYPE_F32>(args, stream);
    default: return HIF8_ERR_INVALID_ARGUMENT;
  }
}

// Fused static quant + linear for m <= 8 rows of FP16/BF16 activations.
template <int OUT, int ASRC>
static int run_fused_linear_out(const GemvArgs &args, cudaStream_t stream) {
  const bool vec_ok = aligned16(args.a) && aligned32(args.w) && args.k % 64 == 0 && args.m <= 8;
  const GemvPlan plan = vec_ok ? plan_gemv_cached(args.m, args.n, args.k, gemv_kernel_ptr<1, OUT, ASRC>())
                               : GemvPlan{};
  if (plan.s == 0) return launch_generic<OUT, ASRC>(args, stream);
  return launch_gemv<1, OUT, ASRC>(args, plan, stream);
}

int run_fused_linear(const GemvArgs &args, int x_dtype, int output_dtype, cudaStream_t stream) {
  const bool bf16_in = x_dtype == HIF8_DTYPE_BF16;
  switch (output_dtype) {
    case HIF8_DTYPE_BF16:
      return bf16_in ? run_fused_linear_out<HIF8_DTYPE_BF16, kActBf16>(args, stream)
                     : run_fused_linear_out<HIF8_DTYPE_BF16, kActF16>(args, stream);
    case HIF8_DTYPE_F16:
      return bf16_in ? run_fused_linear_out<HIF8_DTYPE_F16, kActBf16>(args, stream)
                     : run_fused_linear_out<HIF8_DTYPE_F16, kActF16>(args, stream);
    case HIF8_DTYPE_F32:
      return bf16_in ? run_fused_linear_out<HIF8_DTYPE_F32, kActBf16>(args, stream)
                     : run_fused_linear_out<HIF8_DTYPE_F32, kActF16>(args, stream);
    default:
      return HIF8_ERR_INVALID_ARGUMENT;
  }
}

// Glue + static quant + linear for m <= 8 BF16 rows (decode steps of the
// model): only the persistent kernel has the glue prologue, so a shape it
// cannot plan is refused rather than computed another way.
int run_glue_linear(const GemvArgs &args, cudaStream_t stream) {
  const GlueArgs &gl = args.glue;
  if (args.m < 1 || args.m > 8 || args.k % 256 != 0 || !aligned16(args.a) || !aligned32(args.w))
    return HIF8_ERR_INVALID_ARGUMENT;
  if ((gl.aux && !aligned16(gl.aux)) || (gl.norm_w && !aligned16(gl.norm_w)) ||
      (gl.residual_out && !aligned16(gl.residual_out)))
    return HIF8_ERR_INVALID_ARGUMENT;
  switch (gl.kind) {
    case kGlueSiluMul: {
      const GemvPlan plan = plan_gemv_cached(args.m, args.n, args.k, gemv_kernel_ptr<1, HIF8_DTYPE_BF16, kActSiluMul>());
      return plan.s ? launch_gemv<1, HIF8_DTYPE_BF16, kActSiluMul>(args, plan, stream) : HIF8_ERR_INVALID_ARGUMENT;
    }
    case kGlueGateMul: {
      if (!gl.aux) return HIF8_ERR_INVALID_ARGUMENT;
      const GemvPlan plan = plan_gemv_cached(args.m, args.n, args.k, gemv_kernel_ptr<1, HIF8_DTYPE_BF16, kActGateMul>());
      return plan.s ? launch_gemv<1, HIF8_DTYPE_BF16, kActGateMul>(args, plan, stream) : HIF8_ERR_INVALID_ARGUMENT;
    }
    case kGlueRmsNorm: {
      if (!gl.norm_w) return HIF8_ERR_INVALID_ARGUMENT;
      const GemvPlan plan = plan_gemv_cached(args.m, args.n, args.k, gemv_kernel_ptr<1, HIF8_DTYPE_BF16, kActRmsNorm>());
      return plan.s ? launch_gemv<1, HIF8_DTYPE_BF16, kActRmsNorm>(args, plan, stream) : HIF8_ERR_INVALID_ARGUMENT;
    }
    default:
      return HIF8_ERR_INVALID_ARGUMENT;
  }
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
  if (hif8_gemm_tc_supported(m, n, k) && aligned16(activation) && aligned16(weight) && aligned16(out)) {
    if (workspace_bytes < hif8_gemm_tc_workspace(m, n, k) || (!workspace && hif8_gemm_tc_workspace(m, n, k)))
      return HIF8_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return HIF8_ERR_WORKSPACE;  // TMA wants an aligned base
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

extern "C" int hif8_model_glue_linear(const uint16_t *x, const Hif8GlueArgs *glue, int64_t m, int64_t k,
                                      const uint8_t *weight, const float *fixed_scale, const float *channel_scale,
                                      int64_t n, uint16_t *out, void *stream) {
  if (!x || !glue || !weight || !fixed_scale || !channel_scale || !out || m <= 0 || n <= 0 || k <= 0 ||
      n > 0x7FFFFFFFLL || k > 0x7FFFFFFFLL)
    return HIF8_ERR_INVALID_ARGUMENT;
  GemvArgs args{x, weight, fixed_scale, channel_scale, nullptr, out, (int)m, (int)n, (int)k, 0,
                HIF8_DTYPE_NONE, 0};
  args.glue.kind = glue->kind;
  args.glue.aux = glue->aux;
  args.glue.residual_out = glue->residual_out;
  args.glue.norm_w = glue->norm_w;
  args.glue.eps = glue->eps;
  args.glue.one_plus = glue->one_plus;
  return run_glue_linear(args, static_cast<cudaStream_t>(stream));
}

extern "C" int hif8_linear_partial_f32(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                                       const float *channel_scale, int64_t m, int64_t n, int64_t k, float *out,
                                       void *workspace, size_t workspace_bytes, void *stream) {
  int status = validate_linear(activation, weight, token_scale, channel_scale, nullptr, HIF8_DTYPE_NONE,
                               HIF8_DTYPE_BF16, m, n, k, out);
  if (status != HIF8_OK) return status;
  GemvArgs args{activation, weight, token_scale, channel_scale, nullptr, out, (int)m, (int)n, (int)k, 0,
                HIF8_DTYPE_NONE, 1};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (hif8_gemm_tc_supported(m, n, k) && aligned16(activation) && aligned16(weight) && aligned16(out)) {
    if (workspace_bytes < hif8_gemm_tc_workspace(m, n, k) || (!workspace && hif8_gemm_tc_workspace(m, n, k)))
      return HIF8_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return HIF8_ERR_WORKSPACE;
    return hif8_gemm_tc(args, HIF8_DTYPE_F32, workspace, workspace_bytes, s);
  }
  return run_linear(args, HIF8_DTYPE_F32, s);
}

extern "C" int hif8_static_fused_linear_partial_f32(const void *x, int x_dtype, const uint8_t *weight,
                                                    const float *fixed_scale, const float *channel_scale, int64_t m,
                                                    int64_t n, int64_t k, float *out, void *stream) {
  int status = validate_linear(x, weight, fixed_scale, channel_scale, nullptr, HIF8_DTYPE_NONE, HIF8_DTYPE_BF16, m,
                               n, k, out);
  if (status != HIF8_OK) return status;
  if (m > 8) return HIF8_ERR_INVALID_ARGUMENT;
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  GemvArgs args{x, weight, fixed_scale, channel_scale, nullptr, out, (int)m, (int)n, (int)k, 0, HIF8_DTYPE_NONE, 0};
  return run_fused_linear(args, x_dtype, HIF8_DTYPE_F32, static_cast<cudaStream_t>(stream));
}

extern "C" size_t soft_hif8_fused_gemm_workspace_size(int64_t m, int64_t n, int64_t k) {
  (void)n;
  if (m <= 0 || k <= 0) return 0;
  return ((size_t)m * k + 255) / 256 * 256 + ((size_t)m * sizeof(float) + 255) / 256 * 256;
}

extern "C" int soft_hif8_fused_gemm(const void *x, int x_dtype, const uint8_t *weight, const float *channel_scale,
                                    const void *bias, int bias_dtype, int output_dtype, int64_t m, int64_t n,
                                    int64_t k, void *out, void *workspace, size_t workspace_bytes, void *stream) {
  const float *no_scale = channel_scale;  // token scales come from the dynamic quant
  int status = validate_linear(x, weight, no_scale, channel_scale, bias, bias_dtype, output_dtype, m, n, k, out);
  if (status != HIF8_OK) return status;
  if (m > 2) return HIF8_ERR_INVALID_ARGUMENT;  // reference contract: soft_hif8_fused_gemm requires M <= 2
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  const size_t need = soft_hif8_fused_gemm_workspace_size(m, n, k);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return HIF8_ERR_WORKSPACE;
  uint8_t *codes = static_cast<uint8_t *>(workspace);
  float *scales = reinterpret_cast<float *>(codes + ((size_t)m * k + 255) / 256 * 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the scale needs the whole row before any of it is encoded: the dynamic
  // quant launch (it signals the linear's launch at its start), then the GEMV
  status = hif8_dynamic_quant(x, x_dtype, m, k, codes, scales, 1, s);
  if (status != HIF8_OK) return status;
  GemvArgs args{codes, weight, scales, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                bias ? bias_dtype : HIF8_DTYPE_NONE, 1};
  return run_linear(args, output_dtype, s);
}

static size_t round256(size_t bytes) { return (bytes + 255) / 256 * 256; }

extern "C" size_t hif8_static_linear_workspace_size(int64_t m, int64_t n, int64_t k, int fused_max_rows) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  if (m <= fused_max_rows && m <= 4) return 0;
  return round256((size_t)m * k) + round256((size_t)m * sizeof(float)) + soft_hif8_gemm_workspace_size(m, n, k);
}

extern "C" int hif8_static_linear(const void *x, int x_dtype, const uint8_t *weight, const float *input_scale,
                                  const float *channel_scale, const void *bias, int bias_dtype, int output_dtype,
                                  int64_t m, int64_t n, int64_t k, int fused_max_rows, void *out, void *workspace,
                                  size_t workspace_bytes, void *stream) {
  int status = validate_linear(x, weight, input_scale, channel_scale, bias, bias_dtype, output_dtype, m, n, k, out);
  if (status != HIF8_OK) return status;
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (m <= fused_max_rows && m <= 4) {
    GemvArgs args{x, weight, input_scale, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                  bias ? bias_dtype : HIF8_DTYPE_NONE, 0};
    return run_fused_linear(args, x_dtype, output_dtype, s);
  }
  const size_t need = hif8_static_linear_workspace_size(m, n, k, fused_max_rows);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return HIF8_ERR_WORKSPACE;
  if (hif8_gemm_tc_supported(m, n, k) && aligned16(x) && aligned16(weight) && aligned16(out)) {
    // prefill: the static quant happens in the GEMM's operand pass (FP16/BF16
    // -> decoded static code as BF16), the bytes never reach memory
    GemvArgs args{x, weight, input_scale, channel_scale, bias, out, (int)m, (int)n, (int)k, 0,
                  bias ? bias_dtype : HIF8_DTYPE_NONE, 0};
    return hif8_gemm_tc(args, output_dtype, workspace, workspace_bytes, s, x_dtype);
  }
  uint8_t *codes = static_cast<uint8_t *>(workspace);
  float *row_scale = reinterpret_cast<float *>(codes + round256((size_t)m * k));
  uint8_t *gemm_ws = reinterpret_cast<uint8_t *>(row_scale) + round256((size_t)m * sizeof(float));
  status = hif8_static_quant(x, x_dtype, m, k, input_scale, 1, codes, row_scale, s);
  if (status != HIF8_OK) return status;
  return soft_hif8_gemm(codes, weight, row_scale, channel_scale, bias, bias_dtype, output_dtype, m, n, k, out,
                        gemm_ws, workspace_bytes - (size_t)(gemm_ws - codes), s);
}
