// Activation static quantisation and scaled decode (HBM-streaming kernels).
//
// hif8_static_quant: data = enc_sat(fp32(x) / s), bit-exact with
// calibration.static_quantize_tensor (reference calibration.py:182-201).
// The quotient is formed as x * (1/s) (both correctly rounded, so within two
// units in the last place of the exact quotient); the HiF8 code depends only
// on the exponent and the top four mantissa bits, so whenever the low 19
// mantissa bits of that product are at least 4 units away from a multiple of
// 2^19 the exact IEEE quotient has the same code.  Otherwise -- and for
// overflow, NaN/Inf, or a denormal reciprocal -- the kernel recomputes the
// quotient with the correctly rounded division __fdiv_rn.
#include "hif8_common.cuh"

namespace hif8 {

__device__ __forceinline__ uint32_t quant_one(float f, float s, float r, bool exact_only,
                                              const uint8_t *__restrict__ tbl) {
  float q = __fmul_rn(f, r);
  uint32_t u = __float_as_uint(q);
  const uint32_t low = u & 0x7FFFFu;
  if (exact_only | ((low - 4u) > 0x7FFF8u) | ((u & 0x7F800000u) >= 0x7D000000u)) {
    q = __fdiv_rn(f, s);
    u = __float_as_uint(q);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x80u;
  }
  return tbl[u >> 19];
}

__device__ __forceinline__ void load_encode_table(uint8_t *smem) {
  const uint4 *src = reinterpret_cast<const uint4 *>(g_static_encode.v);
  uint4 *dst = reinterpret_cast<uint4 *>(smem);
  for (int i = threadIdx.x; i < 8192 / 16; i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ float reciprocal(float s, bool &exact_only) {
  const float r = __frcp_rn(s);
  const uint32_t e = __float_as_uint(r) & 0x7F800000u;
  exact_only = (e == 0u) | (e == 0x7F800000u);
  return r;
}

// 16 elements per thread and iteration: two 16-byte loads, one 16-byte store.
__device__ __forceinline__ void write_row_scale(const float *__restrict__ scale, int64_t scale_count,
                                                float *__restrict__ row_scale, int64_t rows) {
  if (!row_scale) return;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x)
    row_scale[r] = scale[r % scale_count];
}

template <int kDtype>
__global__ void __launch_bounds__(256) static_quant_vec16(const uint16_t *__restrict__ x, int64_t k,
                                                          const float *__restrict__ scale,
                                                          int64_t scale_count, uint8_t *__restrict__ out,
                                                          int64_t chunks, float *__restrict__ row_scale,
                                                          int64_t rows) {
  __shared__ __align__(16) uint8_t tbl[8192];
  load_encode_table(tbl);
  pdl_wait();  // x and scale may come from the previous kernel of the stream
  // Let the dependent linear launch now: its CTAs take the SMs this small
  // grid leaves idle and build their tables, then wait for this grid to
  // complete before reading its bytes (measured: the configs[1] step 358.9
  // -> 354.7 us, identical results).
  pdl_launch_dependents();
  write_row_scale(scale, scale_count, row_scale, rows);
  __syncthreads();
  const int64_t chunks_per_row = k >> 4;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = c / chunks_per_row;
    const float s = __ldg(scale + (scale_count == 1 ? 0 : row % scale_count));
    bool exact_only;
    const float r = reciprocal(s, exact_only);
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (c << 4));
    const uint4 a = __ldcs(src), b = __ldcs(src + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = w[2 * j], hi = w[2 * j + 1];
      const uint32_t c0 = quant_one(half_bits_to_f32<kDtype>(lo & 0xFFFFu), s, r, exact_only, tbl);
      const uint32_t c1 = quant_one(half_bits_to_f32<kDtype>(lo >> 16), s, r, exact_only, tbl);
      const uint32_t c2 = quant_one(half_bits_to_f32<kDtype>(hi & 0xFFFFu), s, r, exact_only, tbl);
      const uint32_t c3 = quant_one(half_bits_to_f32<kDtype>(hi >> 16), s, r, exact_only, tbl);
      o[j] = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
    }
    __stcs(reinterpret_cast<uint4 *>(out + (c << 4)), make_uint4(o[0], o[1], o[2], o[3]));
  }
}

template <int kDtype>
__global__ void __launch_bounds__(256) static_quant_scalar(const uint16_t *__restrict__ x, int64_t k,
                                                           const float *__restrict__ scale,
                                                           int64_t scale_count, uint8_t *__restrict__ out,
                                                           int64_t total, float *__restrict__ row_scale,
                                                           int64_t rows) {
  __shared__ __align__(16) uint8_t tbl[8192];
  load_encode_table(tbl);
  pdl_wait();  // x and scale may come from the previous kernel of the stream
  write_row_scale(scale, scale_count, row_scale, rows);
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / k;
    const float s = __ldg(scale + row % scale_count);
    bool exact_only;
    const float r = reciprocal(s, exact_only);
    out[i] = (uint8_t)quant_one(half_bits_to_f32<kDtype>(x[i]), s, r, exact_only, tbl);
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

// 16 bytes in, 32 bytes out per thread and iteration (rows of k % 16 == 0).
__global__ void __launch_bounds__(256) scaled_decode_vec16(const uint8_t *__restrict__ data, int64_t k,
                                                           int64_t stride, const float *__restrict__ scale,
                                                           uint16_t *__restrict__ out, int64_t chunks) {
  __shared__ float tbl[256];
  load_decode_table(tbl);
  __syncthreads();
  const int64_t per_row = k >> 4;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = c / per_row, col = (c - row * per_row) << 4;
    const float s = __ldg(scale + row);
    const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(data + row * stride + col));
    uint4 o0, o1;
    o0.x = decode_pair(tbl, v.x, 0, s);
    o0.y = decode_pair(tbl, v.x, 16, s);
    o0.z = decode_pair(tbl, v.y, 0, s);
    o0.w = decode_pair(tbl, v.y, 16, s);
    o1.x = decode_pair(tbl, v.z, 0, s);
    o1.y = decode_pair(tbl, v.z, 16, s);
    o1.z = decode_pair(tbl, v.w, 0, s);
    o1.w = decode_pair(tbl, v.w, 16, s);
    uint4 *dst = reinterpret_cast<uint4 *>(out + row * k + col);
    __stcs(dst, o0);
    __stcs(dst + 1, o1);
  }
}

// 4 bytes in, 8 bytes out (rows with k % 4 == 0, e.g. KV rows with the
// 4-byte sidecar between them).
__global__ void __launch_bounds__(256) scaled_decode_vec4(const uint8_t *__restrict__ data, int64_t k,
                                                          int64_t stride, const float *__restrict__ scale,
                                                          uint16_t *__restrict__ out, int64_t chunks) {
  __shared__ float tbl[256];
  load_decode_table(tbl);
  __syncthreads();
  const int64_t per_row = k >> 2;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = c / per_row, col = (c - row * per_row) << 2;
    const float s = __ldg(scale + row);
    const uint32_t v = __ldcs(reinterpret_cast<const unsigned int *>(data + row * stride + col));
    uint2 o;
    o.x = decode_pair(tbl, v, 0, s);
    o.y = decode_pair(tbl, v, 16, s);
    __stcs(reinterpret_cast<uint2 *>(out + row * k + col), o);
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
// VEC: 16 bytes in, 32 bytes out per thread (k % 16 == 0, aligned rows).
template <bool VEC>
__global__ void __launch_bounds__(256) embedding_gather(const uint8_t *__restrict__ weight,
                                                        const float *__restrict__ weight_scale, int64_t vocab,
                                                        int64_t k, const int64_t *__restrict__ ids,
                                                        uint16_t *__restrict__ out, int64_t work,
                                                        int32_t *__restrict__ bad_ids) {
  __shared__ float tbl[256];
  load_decode_table(tbl);  // module data: before the dependency wait
  __syncthreads();
  pdl_wait();  // the ids may come from the previous kernel (the last step's argmax)
  const int64_t per_row = VEC ? k >> 4 : k;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < work; c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = c / per_row, j = c - t * per_row;
    const int64_t id = __ldg(ids + t);
    const bool ok = id >= 0 && id < vocab;
    if (!ok && j == 0 && bad_ids) atomicAdd(bad_ids, 1);
    const float s = ok ? bf16_bits_to_f32(f32_to_bf16_bits(__ldg(weight_scale + id))) : 0.f;
    if constexpr (VEC) {
      uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
      if (ok) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(weight + id * k) + j);
        o0 = make_uint4(decode_pair(tbl, v.x, 0, s), decode_pair(tbl, v.x, 16, s), decode_pair(tbl, v.y, 0, s),
                        decode_pair(tbl, v.y, 16, s));
        o1 = make_uint4(decode_pair(tbl, v.z, 0, s), decode_pair(tbl, v.z, 16, s), decode_pair(tbl, v.w, 0, s),
                        decode_pair(tbl, v.w, 16, s));
      }
      uint4 *dst = reinterpret_cast<uint4 *>(out + t * k) + 2 * j;
      dst[0] = o0;
      dst[1] = o1;
    } else {
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
  if (k % 16 == 0 && aligned16(x) && aligned16(data)) {
    const int64_t chunks = total / 16;
    const int grid = grid_for(chunks, 256);
    return x_dtype == HIF8_DTYPE_BF16
               ? launch_pdl(static_quant_vec16<HIF8_DTYPE_BF16>, dim3(grid), dim3(256), 0, stream, xs, k,
                            fixed_scale, scale_count, data, chunks, row_scale, rows)
               : launch_pdl(static_quant_vec16<HIF8_DTYPE_F16>, dim3(grid), dim3(256), 0, stream, xs, k,
                            fixed_scale, scale_count, data, chunks, row_scale, rows);
  }
  const int grid = grid_for(total, 256);
  return x_dtype == HIF8_DTYPE_BF16
             ? launch_pdl(static_quant_scalar<HIF8_DTYPE_BF16>, dim3(grid), dim3(256), 0, stream, xs, k, fixed_scale,
                          scale_count, data, total, row_scale, rows)
             : launch_pdl(static_quant_scalar<HIF8_DTYPE_F16>, dim3(grid), dim3(256), 0, stream, xs, k, fixed_scale,
                          scale_count, data, total, row_scale, rows);
}

extern "C" int hif8_scaled_decode(const uint8_t *data, int64_t rows, int64_t k, int64_t data_row_stride,
                                  const float *scale, uint16_t *out, void *stream_ptr) {
  if (rows < 0 || k <= 0 || data_row_stride < k || (rows > 0 && (!data || !scale || !out)))
    return HIF8_ERR_INVALID_ARGUMENT;
  if (rows == 0) return HIF8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (k % 16 == 0 && data_row_stride % 16 == 0 && aligned16(data) && aligned16(out)) {
    const int64_t chunks = rows * (k / 16);
    scaled_decode_vec16<<<grid_for(chunks, 256), 256, 0, stream>>>(data, k, data_row_stride, scale, out, chunks);
  } else if (k % 4 == 0 && data_row_stride % 4 == 0 && aligned4(data) && aligned4(out)) {
    const int64_t chunks = rows * (k / 4);
    scaled_decode_vec4<<<grid_for(chunks, 256), 256, 0, stream>>>(data, k, data_row_stride, scale, out, chunks);
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
  if (k % 16 == 0 && aligned16(weight) && aligned16(out)) {
    const int64_t work = n * (k / 16);
    return launch_pdl(embedding_gather<true>, dim3(grid_for(work, 256)), dim3(256), 0, stream, weight, weight_scale,
                      vocab, k, ids, out, work, bad_ids);
  }
  const int64_t work = n * k;
  return launch_pdl(embedding_gather<false>, dim3(grid_for(work, 256)), dim3(256), 0, stream, weight, weight_scale,
                    vocab, k, ids, out, work, bad_ids);
}
