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

struct alignas(16) Table12 {
  uint8_t v[4096];
};

// The positive half of the static-saturating encode (index: exponent field
// and top-4 mantissa bits of |q|); a negative value's code is the same
// magnitude code with bit 7 set, except zero, which has no negative code.
HIF8_HD constexpr Table12 make_static_encode_mag_table() {
  Table12 t{};
  for (uint32_t i = 0; i < 4096u; ++i) t.v[i] = static_encode13(i);
  return t;
}

struct alignas(16) TableFq {
  uint16_t v[4096];
};

// BF16 payload of decode(static code) per magnitude index (the exponent
// field and top-4 mantissa bits of |q|): fake quantisation straight to the
// decoded value, for the prologues that quantise an activation and use it
// decoded.  A negative input's value is this with the sign bit set, except
// zero (code 0 decodes to +0).
HIF8_HD constexpr TableFq make_fake_quant_table() {
  TableFq t{};
  for (uint32_t i = 0; i < 4096u; ++i) t.v[i] = (uint16_t)decode_bf16(static_encode13(i));
  return t;
}

// Device copies of the tables (one per translation unit that uses them).
static __device__ const Table13 g_static_encode = make_static_encode_table();
static __device__ const Table12 g_static_encode_mag = make_static_encode_mag_table();
static __device__ const Table256 g_decode_f32 = make_decode_table_f32();
static __device__ const TableFq g_fake_quant_bf16 = make_fake_quant_table();

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

// Two FP32 values as a BF16 pair (lo in bits 0-15) by the hardware
// round-to-nearest-even conversion.  It equals f32_to_bf16_bits on every
// finite or infinite input that is not an FP32 subnormal; callers keep NaN
// and subnormals away from it (f32_to_bf16_bits canonicalises NaN to 0x7FC0).
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// True when no byte of w is the NaN code 0x80.
__device__ __forceinline__ bool no_nan_code(uint32_t w) {
  const uint32_t x = w ^ 0x80808080u;  // a 0x80 byte becomes a zero byte
  return ((x - 0x01010101u) & ~x & 0x80808080u) == 0u;
}

// A scale whose product with any finite HiF8 value (2^-22 .. 2^15) is a
// normal FP32 or +-Inf: 2^-100 <= |s| < 2^111.
__device__ __forceinline__ bool decode_scale_ok(float s) {
  const uint32_t e = (__float_as_uint(s) >> 23) & 0xFFu;
  return e - 27u < 211u;
}

// ------------------------------------------------- static quantisation --

// Shared-memory copy of g_static_encode_mag (4 KB, 16-byte pieces).
__device__ __forceinline__ void load_encode_mag_table(uint8_t *smem) {
  const uint4 *src = reinterpret_cast<const uint4 *>(g_static_encode_mag.v);
  for (int i = threadIdx.x; i < 4096 / 16; i += blockDim.x) reinterpret_cast<uint4 *>(smem)[i] = src[i];
}

// Exact code of the static quantisation of an FP16/BF16 value f by the fixed
// FP32 scale s, given r64 = RN64(1/s) (__drcp_rn).  The reference forms the
// FP32 quotient RN32(f / s) and encodes it.  f / s is a ratio of an integer
// of at most 11 bits and one of at most 24 bits (times a power of two), so
// when it is not itself an FP32 rounding midpoint it lies at least 2^-49
// (relative) away from every midpoint, and no such ratio is a midpoint
// (that would need a 25-bit odd integer to divide out of the 11-bit
// numerator).  The FP64 product f * r64 is within 2^-52 (relative) of f / s,
// so converting it to FP32 rounds to RN32(f / s) for every f and s --
// zero, infinite and NaN scales included (f * Inf, f * 0 and NaN follow the
// IEEE quotient).  The magnitude code then comes from the table, NaN gives
// 0x80 and a nonzero code takes the quotient's sign.
__device__ __forceinline__ uint32_t static_code_exact(float f, double r64, const uint8_t *__restrict__ mag) {
  const uint32_t v = __float_as_uint((float)((double)f * r64));
  if ((v & 0x7FFFFFFFu) > 0x7F800000u) return 0x80u;
  const uint32_t m = mag[(v >> 19) & 0xFFFu];
  return m == 0u ? 0u : m | ((v >> 24) & 0x80u);
}

// HiF8 code of the static quantisation of f by the fixed scale s with r =
// RN32(1/s) and r64 = RN64(1/s) (exact_only: take the exact path, for a
// reciprocal that is zero or infinite or a scale that is not positive).  The
// product q = f * r is within two units in the last place of the correctly
// rounded quotient RN32(f / s), and the magnitude code is a non-decreasing
// function of the value, so when |q| - 4 ulp and |q| + 4 ulp have the same
// code, RN32(f / s) has it too.  The codes of both ends come from the
// magnitude table (index: exponent field and top-4 mantissa bits), the sign
// is OR'd into bit 7 of a nonzero code.  A quotient within 4 ulp of a code
// boundary, an |q| of 2^123 or more and NaN / Inf take static_code_exact.
// `mag` is the shared-memory copy of g_static_encode_mag: with the sign out
// of the index, a warp's lookups over 8 consecutive binades fall into
// distinct banks.
__device__ __forceinline__ uint32_t static_code(float f, float r, double r64, bool exact_only,
                                                const uint8_t *__restrict__ mag) {
  const uint32_t u = __float_as_uint(__fmul_rn(f, r));
  const uint32_t a = max(u & 0x7FFFFFFFu, 4u);
  // a - 4 >= 0; a + 4 can pass 2^31 only for a NaN, which the check below
  // sends to the exact path: the mask keeps that lookup inside the table
  const uint32_t lo = mag[(a - 4u) >> 19], hi = mag[((a + 4u) >> 19) & 0xFFFu];
  if (exact_only | (lo != hi) | (a >= 0x7D000000u)) return static_code_exact(f, r64, mag);
  return lo == 0u ? 0u : lo | ((u >> 24) & 0x80u);
}

// Bits of Q = RN32(x), x = |f| / s, from the product q = RN32(|f| * r),
// r = RN32(1/s), for a positive scale s in [2^-60, 2^60] (scale_edge_ok)
// and q below 2^123 -- the quotient that the reference's FP32 division
// rounds to, without a division.  q is within 1.5 ulp of x (r's relative
// error is at most 2^-24, the product's rounding adds half an ulp) and Q
// within half an ulp, so Q is q or one of its neighbours: Q is above q
// exactly when x exceeds q by more than half the gap to the next float, and
// below it when x falls short by more than half the gap to the previous one.
// x is never an FP32 midpoint (a dyadic |f| / s has at most 11 significant
// bits: s's odd part would have to divide |f|'s), so the comparisons are
// strict.  They are made on the remainder rho = |f| - q * s (one fused
// multiply-add) against the half gaps times s (exact: s / 2 times a power of
// two): rho is an integer multiple of q's and s's unit products, with fewer
// than 25 significant bits whenever |x - q| <= 1 ulp, so it is exact where it
// meets a threshold, and where it is not exact (|x - q| > 1 ulp) it lies far
// from both thresholds.  The sign of a correctly rounded sum is exact, so
// each test is one more fused multiply-add.  q = 0 gives 0 (its lower gap
// is NaN; an underflowed nonzero x may step up to the smallest subnormal,
// whose code is 0 like every value below 2^-23).
__device__ __forceinline__ uint32_t rn_quotient_bits(float fa, float q, float s, float s_half) {
  const uint32_t a = __float_as_uint(q);
  const float rho = __fmaf_rn(-q, s, fa);
  const float up = __uint_as_float(a + 1u) - q;
  const float dn = q - __uint_as_float(a - 1u);
  const uint32_t above = __fmaf_rn(-up, s_half, rho) > 0.f ? 1u : 0u;
  const uint32_t below = __fmaf_rn(dn, s_half, rho) < 0.f ? 1u : 0u;
  return a + above - below;
}

// True when rn_quotient_bits may be used with scale s: 2^-60 <= s <= 2^60.
__device__ __forceinline__ bool scale_edge_ok(float s) {
  const uint32_t u = __float_as_uint(s);
  return u - 0x21800000u <= 0x5D800000u - 0x21800000u;
}

// Static codes of 16 consecutive FP16/BF16 elements (w: their 8 words,
// element 2i in the low half of w[i]) with a POSITIVE fixed scale s in the
// range of scale_edge_ok (r = RN32(1/s), s_half = s / 2), four codes per
// output word in element order: the table entry of each element's correctly
// rounded quotient (rn_quotient_bits).  Returns false when some product
// reaches 2^123 or is NaN / Inf -- the caller then takes
// static_codes16_exact for the chunk.  Each nonzero code gets its element's
// sign, read straight from the input words.
template <int kDtype>
__device__ __forceinline__ bool static_codes16(const uint32_t (&w)[8], float s, float r, float s_half,
                                               const uint8_t *__restrict__ mag, uint32_t (&out)[4]) {
  uint32_t amax = 0u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t c[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t word = w[2 * j + (e >> 1)];
      float f;
      if constexpr (kDtype == HIF8_DTYPE_BF16) f = __uint_as_float((e & 1) ? (word & 0xFFFF0000u) : (word << 16));
      else f = __half2float(__ushort_as_half((unsigned short)((e & 1) ? (word >> 16) : (word & 0xFFFFu))));
      const float fa = fabsf(f);
      const float q = __fmul_rn(fa, r);
      amax = max(amax, __float_as_uint(q));
      c[e] = mag[(rn_quotient_bits(fa, q, s, s_half) >> 19) & 0xFFFu];
    }
    const uint32_t codes = __byte_perm(__byte_perm(c[0], c[1], 0x0040u), __byte_perm(c[2], c[3], 0x0040u), 0x5410u);
    // bit 7 of every byte: the element's sign (bit 15 of each FP16/BF16)
    const uint32_t signs = __byte_perm(w[2 * j], w[2 * j + 1], 0x7531u);
    // codes are below 0x80, so + 0x7F sets bit 7 of exactly the nonzero ones
    out[j] = codes | (signs & (codes + 0x7F7F7F7Fu) & 0x80808080u);
  }
  return amax < 0x7D000000u;
}

// The 16 codes by static_code_exact.
template <int kDtype>
__device__ __forceinline__ void static_codes16_exact(const uint32_t (&w)[8], double r64,
                                                     const uint8_t *__restrict__ mag, uint32_t (&out)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t v = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t word = w[2 * j + (e >> 1)];
      const uint32_t h = (e & 1) ? (word >> 16) : (word & 0xFFFFu);
      v |= static_code_exact(half_bits_to_f32<kDtype>(h), r64, mag) << (8 * e);
    }
    out[j] = v;
  }
}

// True when s is a positive normal power of two: its reciprocal r is then
// exact, so f * r is the exact quotient f / s rounded once -- RN32(f / s)
// itself, overflow and underflow included.
__device__ __forceinline__ bool scale_is_pow2(float s) {
  const uint32_t u = __float_as_uint(s);
  return (u & 0x007FFFFFu) == 0u && u - 0x00800000u < 0x7F000000u;
}

// Static codes of 16 elements for a power-of-two scale (r = 1 / s exact):
// the product is the correctly rounded quotient, so its table entry is the
// code, with no check (NaN gives 0x80).
template <int kDtype>
__device__ __forceinline__ void static_codes16_pow2(const uint32_t (&w)[8], float r, const uint8_t *__restrict__ mag,
                                                    uint32_t (&out)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t c[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t word = w[2 * j + (e >> 1)];
      float f;
      if constexpr (kDtype == HIF8_DTYPE_BF16) f = __uint_as_float((e & 1) ? (word & 0xFFFF0000u) : (word << 16));
      else f = __half2float(__ushort_as_half((unsigned short)((e & 1) ? (word >> 16) : (word & 0xFFFFu))));
      const uint32_t a = __float_as_uint(__fmul_rn(f, r)) & 0x7FFFFFFFu;
      c[e] = a > 0x7F800000u ? 0x80u : (uint32_t)mag[a >> 19];
    }
    const uint32_t codes = __byte_perm(__byte_perm(c[0], c[1], 0x0040u), __byte_perm(c[2], c[3], 0x0040u), 0x5410u);
    const uint32_t signs = __byte_perm(w[2 * j], w[2 * j + 1], 0x7531u);
    // the NaN code 0x80 keeps bit 7 whatever the sign; other codes are below 0x80
    out[j] = codes | (signs & (codes + 0x7F7F7F7Fu) & 0x80808080u);
  }
}


// BF16 payloads of decode(static code) of 16 FP16/BF16 elements (w: their 8
// words, element 2i in the low half of w[i]) quantised with a POSITIVE
// fixed scale s (scale_edge_ok; r = RN32(1/s), s_half = s / 2), two per
// output word in element order -- the rule of static_codes16 with the
// decoded values looked up directly (`fq`: shared-memory copy of
// g_fake_quant_bf16).  Returns false when some product reaches 2^123 or is
// NaN / Inf (the caller takes the exact path).  A nonzero value takes its
// element's sign from the input word.
template <int kDtype>
__device__ __forceinline__ bool fake_quant16(const uint32_t (&w)[8], float s, float r, float s_half,
                                             const uint16_t *__restrict__ fq, uint32_t (&out)[8]) {
  uint32_t amax = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t v[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float f;
      if constexpr (kDtype == HIF8_DTYPE_BF16) f = __uint_as_float(e ? (w[j] & 0xFFFF0000u) : (w[j] << 16));
      else f = __half2float(__ushort_as_half((unsigned short)(e ? (w[j] >> 16) : (w[j] & 0xFFFFu))));
      const float fa = fabsf(f);
      const float q = __fmul_rn(fa, r);
      amax = max(amax, __float_as_uint(q));
      v[e] = fq[(rn_quotient_bits(fa, q, s, s_half) >> 19) & 0xFFFu];
    }
    const uint32_t pair = v[0] | (v[1] << 16);
    // payloads are below 0x8000: + 0x7FFF sets bit 15 of exactly the nonzero ones
    out[j] = pair | (w[j] & (pair + 0x7FFF7FFFu) & 0x80008000u);
  }
  return amax < 0x7D000000u;
}

// Lane-replicated FP32 decode table in shared memory (32 KB): entry b of
// lane l is the word at (b << 5) | l, so every lane reads its own bank and a
// warp's 32 lookups are one wavefront whatever the codes.
constexpr int kLaneDecodeWords = 256 * 32;

__device__ __forceinline__ void load_lane_decode_table(float *smem) {
  for (int i = threadIdx.x; i < kLaneDecodeWords; i += blockDim.x)
    smem[i] = __uint_as_float(g_decode_f32.v[i >> 5]);
}

__device__ __forceinline__ float lane_decode(const float *tbl, uint32_t code, uint32_t lane) {
  return tbl[(code << 5) | lane];
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
