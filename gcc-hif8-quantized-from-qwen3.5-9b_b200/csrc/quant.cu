// Activation static quantisation and scaled decode (HBM-streaming kernels).
//
// hif8_static_quant: data = enc_sat(fp32(x) / s), bit-exact with
// calibration.static_quantize_tensor (reference calibration.py:182-201); the
// per-element rule (a product with the reciprocal, the correctly rounded
// division near code boundaries) is static_code in hif8_common.cuh.
#include "hif8_common.cuh"

namespace hif8 {

__device__ __forceinline__ uint32_t quant_one(float f, float r, double r64, bool exact_only,
                                              const uint8_t *__restrict__ tbl) {
  return static_code(f, r, r64, exact_only, tbl);
}

__device__ __forceinline__ void load_encode_table(uint8_t *smem) { load_encode_mag_table(smem); }

// RN32(1/s) and RN64(1/s); exact_only (every element by the exact FP64
// path) for a reciprocal that is zero, infinite or NaN, and for a scale that
// is not positive (the chunk path reads each code's sign from its input).
__device__ __forceinline__ float reciprocal(float s, bool &exact_only, double &r64) {
  const float r = __frcp_rn(s);
  const uint32_t e = __float_as_uint(r) & 0x7F800000u;
  exact_only = (e == 0u) | (e == 0x7F800000u) | !(s > 0.f);
  r64 = __drcp_rn((double)s);
  return r;
}

__device__ __forceinline__ void write_row_scale(const float *__restrict__ scale, int64_t scale_count,
                                                float *__restrict__ row_scale, int64_t rows) {
  if (!row_scale) return;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x)
    row_scale[r] = scale[r % scale_count];
}

// 16 elements (two 16-byte loads, one 16-byte store) per chunk; every thread
// keeps kQuantUnroll chunks in flight (all loads issued before any
// arithmetic), so the kernel streams at the HBM rate instead of waiting one
// load latency per chunk.  The reciprocal of the fixed scale is formed once
// per thread (kPerRow: once per change of the scale along the thread's
// chunks), and a chunk's row is a 32-bit division only when scales differ
// per row (chunks < 2^32, checked by the launcher).
constexpr int kQuantUnroll = 2;

// The scale's encode mode: kModeQuotient (the correctly rounded quotient
// from the product, static_codes16), kModePow2 (power of two: the product is
// the quotient), kModeExact (every element by the exact FP64 path: zero,
// negative and non-finite scales, and scales outside [2^-60, 2^60]).
struct QuantScale {
  float s, r, s_half;
  double r64;
  int mode;
};
constexpr int kModeQuotient = 0, kModePow2 = 1, kModeExact = 2;

__device__ __forceinline__ QuantScale quant_scale(float s) {
  QuantScale q;
  bool exact_only;
  q.s = s;
  q.s_half = 0.5f * s;
  q.r = reciprocal(s, exact_only, q.r64);
  q.mode = exact_only || !scale_edge_ok(s) ? kModeExact : (scale_is_pow2(s) ? kModePow2 : kModeQuotient);
  return q;
}

template <int kDtype>
__device__ __forceinline__ uint4 quant_chunk(const uint4 a, const uint4 b, const QuantScale &q,
                                             const uint8_t *__restrict__ tbl) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t o[4];
  if (q.mode == kModePow2) {
    static_codes16_pow2<kDtype>(w, q.r, tbl, o);
  } else if (q.mode == kModeExact || !static_codes16<kDtype>(w, q.s, q.r, q.s_half, tbl, o)) {
    // a huge or non-finite product in the chunk (or an extreme scale)
    static_codes16_exact<kDtype>(w, q.r64, tbl, o);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int kDtype, bool kPerRow>
__global__ void __launch_bounds__(256, 4) static_quant_vec16(const uint16_t *__restrict__ x, int64_t k,
                                                          const float *__restrict__ scale,
                                                          int64_t scale_count, uint8_t *__restrict__ out,
                                                          int64_t chunks, float *__restrict__ row_scale,
                                                          int64_t rows) {
  __shared__ __align__(16) uint8_t tbl[4096];
  load_encode_table(tbl);
  pdl_wait();  // x and scale may come from the previous kernel of the stream
  // Let the dependent linear launch now: its CTAs take the SMs this small
  // grid leaves idle and build their tables, then wait for this grid to
  // complete before reading its bytes (measured: the configs[1] step 358.9
  // -> 354.7 us, identical results).
  pdl_launch_dependents();
  write_row_scale(scale, scale_count, row_scale, rows);
  __syncthreads();
  const uint32_t chunks_per_row = (uint32_t)(k >> 4);
  int64_t cur = 0;  // scale index of s / r
  QuantScale qs = quant_scale(__ldg(scale));
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c0 < chunks; c0 += kQuantUnroll * stride) {
    uint4 a[kQuantUnroll], b[kQuantUnroll];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      if (c < chunks) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + (c << 4));
        a[u] = __ldcs(src);
        b[u] = __ldcs(src + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      if (c >= chunks) break;
      if constexpr (kPerRow) {
        const int64_t sidx = (int64_t)((uint32_t)c / chunks_per_row) % scale_count;
        if (sidx != cur) {
          cur = sidx;
          qs = quant_scale(__ldg(scale + sidx));
        }
      }
      __stcs(reinterpret_cast<uint4 *>(out + (c << 4)), quant_chunk<kDtype>(a[u], b[u], qs, tbl));
    }
  }
}

template <int kDtype>
__global__ void __launch_bounds__(256) static_quant_scalar(const uint16_t *__restrict__ x, int64_t k,
                                                           const float *__restrict__ scale,
                                                           int64_t scale_count, uint8_t *__restrict__ out,
                                                           int64_t total, float *__restrict__ row_scale,
                                                           int64_t rows) {
  __shared__ __align__(16) uint8_t tbl[4096];
  load_encode_table(tbl);
  pdl_wait();  // x and scale may come from the previous kernel of the stream
  write_row_scale(scale, scale_count, row_scale, rows);
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / k;
    const float s = __ldg(scale + row % scale_count);
    bool exact_only;
    double r64;
    const float r = reciprocal(s, exact_only, r64);
    out[i] = (uint8_t)quant_one(half_bits_to_f32<kDtype>(x[i]), r, r64, exact_only, tbl);
  }
}

// ---------------------------------------------------------- dynamic quant
//
// hif8_dynamic_quant (reference csrc/opp/op_kernel/hif8_dynamic_quant.cpp
// :11-221; CPU rule codec.py:205-255): per row, scale = max(amax of the
// row's finite |x|, 1e-12) and data = encode(x / scale), NaN / Inf keeping
// their codes.  The amax is the largest 15-bit magnitude pattern below the
// Inf/NaN exponent (the patterns of non-negative values order like the
// values).  |x / scale| <= 1 for finite x, so the static-saturating rule of
// static_code gives the plain encode here.  When the scale is the row's
// amax -- one of its own FP16/BF16 values, at most 11 significant bits --
// the exact quotient x / scale is either a HiF8 code boundary itself or at
// least 2^-17 (relative) away from every boundary (a boundary has at most 5
// significant bits), so the FP32 quotient has the code of the reference's
// double-precision division.  A row whose finite amax is at most 1e-12 is
// divided by the floor 1e-12, which the reference's CPU rule applies as the
// double nearest 1e-12 (not its FP32 rounding, the row scale it stores):
// those rows take the codes of the double quotient (code_of_double).  One
// CTA per row (grid-stride), the row held in registers up to 16384 values.
constexpr int kDynThreads = 256;
constexpr int kDynKeep = 4;  // 16-value chunks per thread held in registers
constexpr double kDynFloorScale = 1.0e-12;
constexpr float kDynFloorScaleF = 1.0e-12f;

// HiF8 code (nearest, ties away) of a double q.  The code boundaries are
// FP32 values, so RN32(q) has q's code unless |q| is below |RN32(q)|: then
// no boundary lies strictly between them, and the FP32 value just below
// RN32(q) in magnitude has q's code (a boundary itself takes the code above
// it, as q does when RN32(q) is the next value up).
__device__ __forceinline__ uint32_t code_of_double(double q, const uint8_t *__restrict__ mag) {
  const float qf = (float)q;
  uint32_t v = __float_as_uint(qf);
  if ((v & 0x7FFFFFFFu) > 0x7F800000u) return 0x80u;
  if (fabs(q) < (double)fabsf(qf)) v -= 1u;  // |qf| > 0 here: the sign bit stays
  const uint32_t m = mag[(v >> 19) & 0xFFFu];
  return m == 0u ? 0u : m | ((v >> 24) & 0x80u);
}

// The 16 codes of a chunk of a floor-scale row.
template <int kDtype>
__device__ __forceinline__ uint4 floor_chunk(const uint4 a, const uint4 b, const uint8_t *__restrict__ tbl) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t o[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const uint32_t h = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    o[e >> 2] |= code_of_double((double)half_bits_to_f32<kDtype>(h) / kDynFloorScale, tbl) << (8 * (e & 3));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int kDtype>
__device__ __forceinline__ uint32_t finite_mag_max16(const uint4 a, const uint4 b, uint32_t m) {
  constexpr uint32_t kInf = kDtype == HIF8_DTYPE_BF16 ? 0x7F80u : 0x7C00u;
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lo = w[j] & 0x7FFFu, hi = (w[j] >> 16) & 0x7FFFu;
    m = max(m, lo < kInf ? lo : 0u);
    m = max(m, hi < kInf ? hi : 0u);
  }
  return m;
}

template <int kDtype>
__global__ void __launch_bounds__(kDynThreads) dynamic_quant_vec16(const uint16_t *__restrict__ x, int64_t rows,
                                                                   int64_t k, uint8_t *__restrict__ out,
                                                                   float *__restrict__ row_scale,
                                                                   int64_t scale_stride) {
  __shared__ __align__(16) uint8_t tbl[4096];
  __shared__ uint32_t warp_max[kDynThreads / 32];
  load_encode_mag_table(tbl);  // module data: before the dependency wait
  pdl_wait();                  // x may come from the previous kernel of the stream
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunks = k >> 4;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * k);
    uint4 a[kDynKeep], b[kDynKeep];
    uint32_t m = 0;
#pragma unroll
    for (int u = 0; u < kDynKeep; ++u) {
      const int64_t c = tid + (int64_t)u * kDynThreads;
      if (c < chunks) {
        a[u] = __ldcs(xr + 2 * c);
        b[u] = __ldcs(xr + 2 * c + 1);
        m = finite_mag_max16<kDtype>(a[u], b[u], m);
      }
    }
    for (int64_t c = tid + (int64_t)kDynKeep * kDynThreads; c < chunks; c += kDynThreads)
      m = finite_mag_max16<kDtype>(__ldg(xr + 2 * c), __ldg(xr + 2 * c + 1), m);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if (lane == 0) warp_max[warp] = m;
    __syncthreads();
    m = 0;
#pragma unroll
    for (int w = 0; w < kDynThreads / 32; ++w) m = max(m, warp_max[w]);
    const float amax = half_bits_to_f32<kDtype>(m);
    const bool floor_row = !(amax > kDynFloorScaleF);
    const float s = floor_row ? kDynFloorScaleF : amax;
    if (tid == 0 && row_scale) row_scale[row * scale_stride] = s;
    const QuantScale qs = quant_scale(s);
    uint4 *orow = reinterpret_cast<uint4 *>(out + row * k);
#pragma unroll
    for (int u = 0; u < kDynKeep; ++u) {
      const int64_t c = tid + (int64_t)u * kDynThreads;
      if (c < chunks)
        __stcs(orow + c, floor_row ? floor_chunk<kDtype>(a[u], b[u], tbl)
                                   : quant_chunk<kDtype>(a[u], b[u], qs, tbl));
    }
    for (int64_t c = tid + (int64_t)kDynKeep * kDynThreads; c < chunks; c += kDynThreads) {
      const uint4 a1 = __ldg(xr + 2 * c), b1 = __ldg(xr + 2 * c + 1);
      __stcs(orow + c, floor_row ? floor_chunk<kDtype>(a1, b1, tbl)
                                 : quant_chunk<kDtype>(a1, b1, qs, tbl));
    }
    __syncthreads();  // warp_max is rewritten by the next row
  }
}

// Any k and alignment: one CTA per row, one value per thread and step.
template <int kDtype>
__global__ void __launch_bounds__(kDynThreads) dynamic_quant_scalar(const uint16_t *__restrict__ x, int64_t rows,
                                                                    int64_t k, uint8_t *__restrict__ out,
                                                                    float *__restrict__ row_scale,
                                                                    int64_t scale_stride) {
  __shared__ __align__(16) uint8_t tbl[4096];
  __shared__ uint32_t warp_max[kDynThreads / 32];
  load_encode_mag_table(tbl);
  pdl_wait();
  constexpr uint32_t kInf = kDtype == HIF8_DTYPE_BF16 ? 0x7F80u : 0x7C00u;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint16_t *xr = x + row * k;
    uint32_t m = 0;
    for (int64_t c = tid; c < k; c += kDynThreads) {
      const uint32_t mag = xr[c] & 0x7FFFu;
      m = max(m, mag < kInf ? mag : 0u);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if (lane == 0) warp_max[warp] = m;
    __syncthreads();
    m = 0;
#pragma unroll
    for (int w = 0; w < kDynThreads / 32; ++w) m = max(m, warp_max[w]);
    const float amax = half_bits_to_f32<kDtype>(m);
    const bool floor_row = !(amax > kDynFloorScaleF);
    const float s = floor_row ? kDynFloorScaleF : amax;
    if (tid == 0 && row_scale) row_scale[row * scale_stride] = s;
    bool exact_only;
    double r64;
    const float r = reciprocal(s, exact_only, r64);
    for (int64_t c = tid; c < k; c += kDynThreads) {
      const float f = half_bits_to_f32<kDtype>(xr[c]);
      out[row * k + c] = (uint8_t)(floor_row ? code_of_double((double)f / kDynFloorScale, tbl)
                                             : quant_one(f, r, r64, exact_only, tbl));
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ scaled decode

__device__ __forceinline__ void load_decode_table(float *smem) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) smem[i] = __uint_as_float(g_decode_f32.v[i]);
}

__device__ __forceinline__ uint32_t decode_pair(const float *tbl, uint32_t word, int shift, float s) {
  const uint32_t lo = f32_to_bf16_bits(tbl[(word >> shift) & 0xFFu] * s);
  const uint32_t hi = f32_to_bf16_bits(tbl[(word >> (shift + 8)) & 0xFFu] * s);
  return lo | (hi << 16);
}

// The same through the lane-replicated table (conflict-free lookups).
__device__ __forceinline__ uint32_t lane_decode_pair(const float *tbl, uint32_t word, int shift, float s,
                                                     uint32_t lane) {
  const uint32_t lo = f32_to_bf16_bits(lane_decode(tbl, (word >> shift) & 0xFFu, lane) * s);
  const uint32_t hi = f32_to_bf16_bits(lane_decode(tbl, (word >> (shift + 8)) & 0xFFu, lane) * s);
  return lo | (hi << 16);
}

__device__ __forceinline__ uint4 lane_decode16(const float *tbl, const uint32_t (&w)[4], float s, uint32_t lane,
                                               int half) {
  return make_uint4(lane_decode_pair(tbl, w[2 * half], 0, s, lane), lane_decode_pair(tbl, w[2 * half], 16, s, lane),
                    lane_decode_pair(tbl, w[2 * half + 1], 0, s, lane),
                    lane_decode_pair(tbl, w[2 * half + 1], 16, s, lane));
}

// The pair through the hardware BF16 conversion (callers: no NaN code in the
// word and decode_scale_ok(s), so it equals lane_decode_pair).
__device__ __forceinline__ uint32_t lane_decode_pair_hw(const float *tbl, uint32_t word, int shift, float s,
                                                        uint32_t lane) {
  return bf16x2_rn(lane_decode(tbl, (word >> shift) & 0xFFu, lane) * s,
                   lane_decode(tbl, (word >> (shift + 8)) & 0xFFu, lane) * s);
}

// 16 bytes -> 32 bytes (two uint4 of BF16 pairs): the hardware conversion
// when the chunk allows it, else the exact-NaN software rounding.
__device__ __forceinline__ void lane_decode_chunk(const float *tbl, const uint32_t (&w)[4], float s, uint32_t lane,
                                                  uint4 &o0, uint4 &o1) {
  if (decode_scale_ok(s) && no_nan_code(w[0]) && no_nan_code(w[1]) && no_nan_code(w[2]) && no_nan_code(w[3])) {
    o0 = make_uint4(lane_decode_pair_hw(tbl, w[0], 0, s, lane), lane_decode_pair_hw(tbl, w[0], 16, s, lane),
                    lane_decode_pair_hw(tbl, w[1], 0, s, lane), lane_decode_pair_hw(tbl, w[1], 16, s, lane));
    o1 = make_uint4(lane_decode_pair_hw(tbl, w[2], 0, s, lane), lane_decode_pair_hw(tbl, w[2], 16, s, lane),
                    lane_decode_pair_hw(tbl, w[3], 0, s, lane), lane_decode_pair_hw(tbl, w[3], 16, s, lane));
  } else {
    o0 = lane_decode16(tbl, w, s, lane, 0);
    o1 = lane_decode16(tbl, w, s, lane, 1);
  }
}

// Scaled decode units: 16 bytes in, 32 bytes out (ELEMS = 16, rows of k % 16
// == 0) or 4 bytes in, 8 bytes out (ELEMS = 4, e.g. KV rows with the 4-byte
// sidecar between them).  kDecodeUnroll units per thread in flight, the row
// of a unit a 32-bit division (units < 2^32, checked by the launcher), the
// decode through the lane-replicated table.
constexpr int kDecodeUnroll = 4;

template <int ELEMS>
__global__ void __launch_bounds__(256) scaled_decode_vec(const uint8_t *__restrict__ data, int64_t k,
                                                         int64_t stride, const float *__restrict__ scale,
                                                         uint16_t *__restrict__ out, int64_t chunks) {
  __shared__ float tbl[kLaneDecodeWords];
  load_lane_decode_table(tbl);
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t per_row = (uint32_t)(k / ELEMS);
  const int64_t gstride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c0 < chunks; c0 += kDecodeUnroll * gstride) {
    uint32_t w[kDecodeUnroll][4];
    int64_t row[kDecodeUnroll], col[kDecodeUnroll];
    float sc[kDecodeUnroll];
#pragma unroll
    for (int u = 0; u < kDecodeUnroll; ++u) {
      const int64_t c = c0 + u * gstride;
      row[u] = c < chunks ? (int64_t)((uint32_t)c / per_row) : 0;
      col[u] = (c - row[u] * per_row) * ELEMS;
      w[u][0] = w[u][1] = w[u][2] = w[u][3] = 0;
      sc[u] = 0.f;
      if (c < chunks) {
        sc[u] = __ldg(scale + row[u]);
        if constexpr (ELEMS == 16) {
          const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(data + row[u] * stride + col[u]));
          w[u][0] = v.x;
          w[u][1] = v.y;
          w[u][2] = v.z;
          w[u][3] = v.w;
        } else {
          w[u][0] = __ldcs(reinterpret_cast<const unsigned int *>(data + row[u] * stride + col[u]));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kDecodeUnroll; ++u) {
      const int64_t c = c0 + u * gstride;
      if (c >= chunks) break;
      if constexpr (ELEMS == 16) {
        uint4 *dst = reinterpret_cast<uint4 *>(out + row[u] * k + col[u]);
        uint4 o0, o1;
        lane_decode_chunk(tbl, w[u], sc[u], lane, o0, o1);
        __stcs(dst, o0);
        __stcs(dst + 1, o1);
      } else {
        uint2 o;
        if (decode_scale_ok(sc[u]) && no_nan_code(w[u][0])) {
          o.x = lane_decode_pair_hw(tbl, w[u][0], 0, sc[u], lane);
          o.y = lane_decode_pair_hw(tbl, w[u][0], 16, sc[u], lane);
        } else {
          o.x = lane_decode_pair(tbl, w[u][0], 0, sc[u], lane);
          o.y = lane_decode_pair(tbl, w[u][0], 16, sc[u], lane);
        }
        __stcs(reinterpret_cast<uint2 *>(out + row[u] * k + col[u]), o);
      }
    }
  }
}

__global__ void __launch_bounds__(256) scaled_decode_scalar(const uint8_t *__restrict__ data, int64_t k,
                                                            int64_t stride, const float *__restrict__ scale,
                                                            uint16_t *__restrict__ out, int64_t total) {
  __shared__ float tbl[256];
  load_decode_table(tbl);
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / k, col = i - row * k;
    out[i] = (uint16_t)f32_to_bf16_bits(tbl[data[row * stride + col]] * __ldg(scale + row));
  }
}

// Embedding rows: out[t, j] = bf16_rne(decode(w[ids[t], j]) * bf16_rne(ws[ids[t]]))
// -- the W8A8HIF8_SOFT embedding of the reference (scheme.py:120-131: BF16
// decode table rows times the row scale cast to BF16, a BF16 product).  Both
// factors are BF16 values, so their FP32 product is exact and is rounded
// once.  Ids outside [0, vocab) give a zero row and count into *bad_ids.
// VEC: 16 bytes in, 32 bytes out per unit (k % 16 == 0, aligned rows), and
// kEmbedUnroll units per thread in flight: the id loads of all of them, then
// their scale and row loads, then the decode -- two dependent load latencies
// per kEmbedUnroll units instead of per unit.  A unit's row is a 32-bit
// division (units < 2^32, checked by the launcher).
constexpr int kEmbedUnroll = 4;

template <bool VEC>
__global__ void __launch_bounds__(256) embedding_gather(const uint8_t *__restrict__ weight,
                                                        const float *__restrict__ weight_scale, int64_t vocab,
                                                        int64_t k, const int64_t *__restrict__ ids,
                                                        uint16_t *__restrict__ out, int64_t work,
                                                        int32_t *__restrict__ bad_ids) {
  __shared__ float tbl[VEC ? kLaneDecodeWords : 256];
  if constexpr (VEC) load_lane_decode_table(tbl);  // module data: before the dependency wait
  else load_decode_table(tbl);
  __syncthreads();
  pdl_wait();  // the ids may come from the previous kernel (the last step's argmax)
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if constexpr (VEC) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t per_row = (uint32_t)(k >> 4);
    for (int64_t c0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c0 < work; c0 += kEmbedUnroll * stride) {
      int64_t t[kEmbedUnroll], id[kEmbedUnroll];
      uint32_t j[kEmbedUnroll];
#pragma unroll
      for (int u = 0; u < kEmbedUnroll; ++u) {
        const int64_t c = c0 + u * stride;
        t[u] = c < work ? (int64_t)((uint32_t)c / per_row) : 0;
        j[u] = (uint32_t)(c - t[u] * per_row);
        id[u] = c < work ? __ldg(ids + t[u]) : -1;
      }
      float sc[kEmbedUnroll];
      uint4 v[kEmbedUnroll];
#pragma unroll
      for (int u = 0; u < kEmbedUnroll; ++u) {
        const bool ok = id[u] >= 0 && id[u] < vocab;
        sc[u] = ok ? __ldg(weight_scale + id[u]) : 0.f;
        v[u] = ok ? __ldg(reinterpret_cast<const uint4 *>(weight + id[u] * k) + j[u]) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kEmbedUnroll; ++u) {
        const int64_t c = c0 + u * stride;
        if (c >= work) break;
        const bool ok = id[u] >= 0 && id[u] < vocab;
        if (!ok && j[u] == 0 && bad_ids) atomicAdd(bad_ids, 1);
        const float s = ok ? bf16_bits_to_f32(f32_to_bf16_bits(sc[u])) : 0.f;
        uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
        if (ok) {
          const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
          lane_decode_chunk(tbl, w, s, lane, o0, o1);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(out + t[u] * k) + 2 * j[u];
        __stcs(dst, o0);
        __stcs(dst + 1, o1);
      }
    }
  } else {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < work; c += stride) {
      const int64_t t = c / k, j = c - t * k;
      const int64_t id = __ldg(ids + t);
      const bool ok = id >= 0 && id < vocab;
      if (!ok && j == 0 && bad_ids) atomicAdd(bad_ids, 1);
      const float s = ok ? bf16_bits_to_f32(f32_to_bf16_bits(__ldg(weight_scale + id))) : 0.f;
      out[t * k + j] = ok ? (uint16_t)f32_to_bf16_bits(tbl[weight[id * k + j]] * s) : (uint16_t)0;
    }
  }
}

static int grid_for(int64_t work, int threads) {
  const int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 8;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace hif8

using namespace hif8;

extern "C" int hif8_static_quant(const void *x, int x_dtype, int64_t rows, int64_t k,
                                 const float *fixed_scale, int64_t scale_count, uint8_t *data,
                                 float *row_scale, void *stream_ptr) {
  if (rows < 0 || k <= 0 || scale_count <= 0 || (rows > 0 && (!x || !data)) || !fixed_scale)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  if (rows % scale_count != 0) return HIF8_ERR_INVALID_ARGUMENT;
  if (rows == 0) return HIF8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const uint16_t *xs = static_cast<const uint16_t *>(x);
  const int64_t total = rows * k;
  if (k % 16 == 0 && aligned16(x) && aligned16(data) && total / 16 <= 0xFFFFFFFFLL) {
    const int64_t chunks = total / 16;
    // one chunk per thread up to 8 CTAs per SM; beyond that wave each thread
    // walks its chunks kQuantUnroll at a time
    const int grid = grid_for(chunks, 256);
    const bool bf16 = x_dtype == HIF8_DTYPE_BF16;
    if (scale_count == 1)
      return bf16 ? launch_pdl(static_quant_vec16<HIF8_DTYPE_BF16, false>, dim3(grid), dim3(256), 0, stream, xs, k,
                               fixed_scale, scale_count, data, chunks, row_scale, rows)
                  : launch_pdl(static_quant_vec16<HIF8_DTYPE_F16, false>, dim3(grid), dim3(256), 0, stream, xs, k,
                               fixed_scale, scale_count, data, chunks, row_scale, rows);
    return bf16 ? launch_pdl(static_quant_vec16<HIF8_DTYPE_BF16, true>, dim3(grid), dim3(256), 0, stream, xs, k,
                             fixed_scale, scale_count, data, chunks, row_scale, rows)
                : launch_pdl(static_quant_vec16<HIF8_DTYPE_F16, true>, dim3(grid), dim3(256), 0, stream, xs, k,
                             fixed_scale, scale_count, data, chunks, row_scale, rows);
  }
  const int grid = grid_for(total, 256);
  return x_dtype == HIF8_DTYPE_BF16
             ? launch_pdl(static_quant_scalar<HIF8_DTYPE_BF16>, dim3(grid), dim3(256), 0, stream, xs, k, fixed_scale,
                          scale_count, data, total, row_scale, rows)
             : launch_pdl(static_quant_scalar<HIF8_DTYPE_F16>, dim3(grid), dim3(256), 0, stream, xs, k, fixed_scale,
                          scale_count, data, total, row_scale, rows);
}

extern "C" int hif8_dynamic_quant(const void *x, int x_dtype, int64_t rows, int64_t k, uint8_t *data,
                                  float *row_scale, int64_t scale_stride, void *stream_ptr) {
  if (rows < 0 || k <= 0 || scale_stride < 1 || (rows > 0 && (!x || !data || !row_scale)))
    return HIF8_ERR_INVALID_ARGUMENT;
  if (x_dtype != HIF8_DTYPE_F16 && x_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  if (rows == 0) return HIF8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const uint16_t *xs = static_cast<const uint16_t *>(x);
  const int64_t cap = (int64_t)num_sms() * 8;
  const dim3 grid((unsigned)(rows < cap ? rows : cap));
  const bool bf16 = x_dtype == HIF8_DTYPE_BF16;
  if (k % 16 == 0 && aligned16(x) && aligned16(data))
    return bf16 ? launch_pdl(dynamic_quant_vec16<HIF8_DTYPE_BF16>, grid, dim3(kDynThreads), 0, stream, xs, rows, k,
                             data, row_scale, scale_stride)
                : launch_pdl(dynamic_quant_vec16<HIF8_DTYPE_F16>, grid, dim3(kDynThreads), 0, stream, xs, rows, k,
                             data, row_scale, scale_stride);
  return bf16 ? launch_pdl(dynamic_quant_scalar<HIF8_DTYPE_BF16>, grid, dim3(kDynThreads), 0, stream, xs, rows, k,
                           data, row_scale, scale_stride)
              : launch_pdl(dynamic_quant_scalar<HIF8_DTYPE_F16>, grid, dim3(kDynThreads), 0, stream, xs, rows, k,
                           data, row_scale, scale_stride);
}

extern "C" int hif8_scaled_decode(const uint8_t *data, int64_t rows, int64_t k, int64_t data_row_stride,
                                  const float *scale, uint16_t *out, void *stream_ptr) {
  if (rows < 0 || k <= 0 || data_row_stride < k || (rows > 0 && (!data || !scale || !out)))
    return HIF8_ERR_INVALID_ARGUMENT;
  if (rows == 0) return HIF8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (k % 16 == 0 && data_row_stride % 16 == 0 && aligned16(data) && aligned16(out) &&
      rows * (k / 16) <= 0xFFFFFFFFLL) {
    const int64_t chunks = rows * (k / 16);
    scaled_decode_vec<16><<<grid_for(chunks, 256), 256, 0, stream>>>(
        data, k, data_row_stride, scale, out, chunks);
  } else if (k % 4 == 0 && data_row_stride % 4 == 0 && aligned4(data) && aligned4(out) &&
             rows * (k / 4) <= 0xFFFFFFFFLL) {
    const int64_t chunks = rows * (k / 4);
    scaled_decode_vec<4><<<grid_for(chunks, 256), 256, 0, stream>>>(
        data, k, data_row_stride, scale, out, chunks);
  } else {
    const int64_t total = rows * k;
    scaled_decode_scalar<<<grid_for(total, 256), 256, 0, stream>>>(data, k, data_row_stride, scale, out, total);
  }
  return check_launch();
}

extern "C" int hif8_embedding_gather(const uint8_t *weight, const float *weight_scale, int64_t vocab, int64_t k,
                                     const int64_t *ids, int64_t n, uint16_t *out, int32_t *bad_ids,
                                     void *stream_ptr) {
  if (vocab <= 0 || k <= 0 || n < 0 || (n > 0 && (!weight || !weight_scale || !ids || !out)))
    return HIF8_ERR_INVALID_ARGUMENT;
  if (n == 0) return HIF8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (k % 16 == 0 && aligned16(weight) && aligned16(out) && n * (k / 16) <= 0xFFFFFFFFLL) {
    const int64_t work = n * (k / 16);
    return launch_pdl(embedding_gather<true>, dim3(grid_for(work, 256)),
                      dim3(256), 0, stream, weight, weight_scale, vocab, k, ids, out, work, bad_ids);
  }
  const int64_t work = n * k;
  return launch_pdl(embedding_gather<false>, dim3(grid_for(work, 256)), dim3(256), 0, stream, weight, weight_scale,
                    vocab, k, ids, out, work, bad_ids);
}
