// Paged HiF8 KV cache: fused static write, paged attention that decodes only
// the touched pages, and the dense gather-decode of kv_runtime._gather_dense_hif8.
//
// Page layout (reference src/vllm_ascend_hif8/kv_cache.py:26-88): a cache is
// [num_blocks, block_size, kv_heads, head_size + 4] bytes; each row holds
// head_size HiF8 codes followed by the row's little-endian FP32 scale.
#include <math_constants.h>

#include "hif8_common.cuh"

namespace hif8 {

// ------------------------------------------------------------ KV write ---

__device__ __forceinline__ uint32_t kv_quant_one(float f, float s, float r, bool exact_only,
                                                 const uint8_t *__restrict__ tbl) {
  float q = __fmul_rn(f, r);
  uint32_t u = __float_as_uint(q);
  const uint32_t low = u & 0x7FFFFu;
  if (exact_only | ((low - 4u) > 0x7FFF8u) | ((u & 0x7F800000u) >= 0x7D000000u)) {
    q = __fdiv_rn(f, s);  // correctly rounded quotient near a code boundary
    u = __float_as_uint(q);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x80u;
  }
  return tbl[u >> 19];
}

struct KvWriteArgs {
  const uint16_t *src[2];  // key, value: [tokens, heads, D] with token stride
  const float *scale[2];   // per head
  uint8_t *cache[2];
  const int64_t *slots;
  int32_t *bad_slots;
  int64_t tokens, heads, d, token_stride, num_blocks, block_size;
  int planes;  // 1 = K only, 2 = K and V
};

// One warp per (plane, token, head) row: 4 elements per lane and step, packed
// into one 4-byte store; lane 0 appends the FP32 scale.
template <int kDtype>
__global__ void __launch_bounds__(256) kv_write_kernel(const KvWriteArgs p) {
  pdl_wait();  // inputs come from the previous kernel of the stream
  __shared__ __align__(16) uint8_t tbl[8192];
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(g_static_encode.v);
    for (int i = threadIdx.x; i < 512; i += blockDim.x) reinterpret_cast<uint4 *>(tbl)[i] = src[i];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t rows = p.tokens * p.heads;
  const int64_t total = rows * p.planes;
  const int64_t width = p.d + 4;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < total;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int plane = (int)(row / rows);
    const int64_t rr = row - plane * rows;
    const int64_t tok = rr / p.heads, h = rr - tok * p.heads;
    const int64_t slot = p.slots[tok];
    if (slot < 0) continue;
    const int64_t block = slot / p.block_size, off = slot - block * p.block_size;
    if (block >= p.num_blocks) {
      if (lane == 0 && p.bad_slots && plane == 0 && h == 0) atomicAdd(p.bad_slots, 1);
      continue;
    }
    const float s = p.scale[plane][h];
    const float r = __frcp_rn(s);
    const uint32_t re = __float_as_uint(r) & 0x7F800000u;
    const bool exact_only = (re == 0u) | (re == 0x7F800000u);
    const uint16_t *src = p.src[plane] + tok * p.token_stride + h * p.d;
    uint8_t *dst = p.cache[plane] + ((block * p.block_size + off) * p.heads + h) * width;
    for (int64_t c = lane * 4; c < p.d; c += 128) {
      const uint2 v = *reinterpret_cast<const uint2 *>(src + c);
      const uint32_t b0 = kv_quant_one(half_bits_to_f32<kDtype>(v.x & 0xFFFFu), s, r, exact_only, tbl);
      const uint32_t b1 = kv_quant_one(half_bits_to_f32<kDtype>(v.x >> 16), s, r, exact_only, tbl);
      const uint32_t b2 = kv_quant_one(half_bits_to_f32<kDtype>(v.y & 0xFFFFu), s, r, exact_only, tbl);
      const uint32_t b3 = kv_quant_one(half_bits_to_f32<kDtype>(v.y >> 16), s, r, exact_only, tbl);
      *reinterpret_cast<uint32_t *>(dst + c) = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
    if (lane == 0) *reinterpret_cast<float *>(dst + p.d) = s;
  }
}

// ------------------------------------------------------ paged attention ---

constexpr int kAttnChunk = 256;  // keys per CTA (one per thread in the score phase)
constexpr int kAttnThreads = 256;

struct AttnArgs {
  const uint16_t *q;          // [tokens, heads, D] BF16
  const uint8_t *kc, *vc;     // caches
  const int32_t *tables;      // [batch, max_blocks]
  const int32_t *seq_lens;    // [batch]
  const int32_t *q_start;     // [batch + 1]
  uint16_t *out;              // [tokens, heads, D] BF16
  float *part;                // split partials (null when splits == 1)
  int64_t heads, kv_heads, d, block_size, max_blocks, num_blocks;
  int splits;                 // KV chunks per request (grid.y)
  int q_rows_per_cta;         // query rows handled per CTA (grid.z groups)
  float scale;
  int causal;
};

// Page of key position `pos` of a request, or -1 when the block table does
// not cover it or names a block outside the cache (such keys are skipped).
__device__ __forceinline__ int64_t page_of(const int32_t *table, int64_t pos, int64_t block_size,
                                          int64_t max_blocks, int64_t num_blocks) {
  const int64_t col = pos / block_size;
  if (col >= max_blocks) return -1;
  const int64_t blk = table[col];
  return (blk >= 0 && blk < num_blocks) ? blk : -1;
}

// Partial layout per (token, head, split): D floats of unnormalised output,
// then the running max and the sum of exponentials.
__host__ __device__ inline int64_t part_stride(int64_t d) { return d + 2; }

// CTA = (request b, kv head h, KV chunk s, query-row group z).  Query vectors
// NQ = (query rows of the group) x (query heads of the GQA group).
template <int NQ>
__global__ void __launch_bounds__(kAttnThreads) paged_attention_kernel(const AttnArgs p) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x / (int)p.kv_heads, h = blockIdx.x - b * (int)p.kv_heads;
  const int split = blockIdx.y;
  const int D = (int)p.d;
  const int group = (int)(p.heads / p.kv_heads);
  const int q0 = p.q_start[b], q_len = p.q_start[b + 1] - q0;
  const int seq = p.seq_lens[b];
  const int row_begin = blockIdx.z * p.q_rows_per_cta;
  const int rows = min(p.q_rows_per_cta, q_len - row_begin);
  if (rows <= 0) return;
  const int nq = rows * group;  // <= NQ
  const int chunk0 = split * kAttnChunk;

  float *lut = sm;                       // 256
  float *qs = lut + 256;                 // [NQ][D]
  float *probs = qs + NQ * D;            // [kAttnChunk][NQ]
  float *red = probs + kAttnChunk * NQ;  // [2][NQ][8 warps]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 256; i += blockDim.x) lut[i] = __uint_as_float(g_decode_f32.v[i]);
  for (int i = tid; i < NQ * D; i += blockDim.x) {
    const int v = i / D, c = i - v * D;
    float x = 0.f;
    if (v < nq) {
      const int r = v / group, gq = v - r * group;
      const int64_t tok = q0 + row_begin + r;
      x = bf16_bits_to_f32(p.q[(tok * p.heads + (int64_t)h * group + gq) * D + c]);
    }
    qs[i] = x;
  }
  __syncthreads();

  // limit of keys visible to query vector v: causal right-aligned positions
  // key j is visible to query row r (0-based in the request) iff
  // j <= seq - q_len + r.
  const int64_t width = p.d + 4;
  const int64_t head_off = (int64_t)h * width;
  const int32_t *table = p.tables + (int64_t)b * p.max_blocks;

  // ---- scores: thread tid owns key chunk0 + tid -----------------------------
  const int key = chunk0 + tid;
  float logit[NQ];
#pragma unroll
  for (int v = 0; v < NQ; ++v) logit[v] = -CUDART_INF_F;
  const int64_t kblk = key < seq ? page_of(table, key, p.block_size, p.max_blocks, p.num_blocks) : -1;
  if (kblk >= 0) {
    const int64_t blk = kblk;
    const uint8_t *row = p.kc + ((blk * p.block_size + key % p.block_size) * p.kv_heads) * width + head_off;
    const float ks = *reinterpret_cast<const float *>(row + D);
    float acc[NQ];
#pragma unroll
    for (int v = 0; v < NQ; ++v) acc[v] = 0.f;
    for (int c = 0; c < D; c += 4) {
      const uint32_t w = *reinterpret_cast<const uint32_t *>(row + c);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // the reference materialises K as BF16 (decode x scale, rounded)
        const float kv = bf16_bits_to_f32(f32_to_bf16_bits(lut[(w >> (8 * e)) & 0xFFu] * ks));
#pragma unroll
        for (int v = 0; v < NQ; ++v) acc[v] = fmaf(qs[v * D + c + e], kv, acc[v]);
      }
    }
#pragma unroll
    for (int v = 0; v < NQ; ++v) {
      if (v < nq) {
        const int r = v / group;
        const bool visible = !p.causal || key <= seq - q_len + row_begin + r;
        if (visible) logit[v] = acc[v] * p.scale;
      }
    }
  }
  // ---- block max / exp / sum per query vector ------------------------------
  float *red_max = red, *red_sum = red + NQ * 8;
#pragma unroll
  for (int v = 0; v < NQ; ++v) {
    float m = logit[v];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) red_max[v * 8 + warp] = m;
  }
  __syncthreads();
  float mx[NQ];
#pragma unroll
  for (int v = 0; v < NQ; ++v) {
    float m = red_max[v * 8];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red_max[v * 8 + w]);
    mx[v] = m;
    const float e = (logit[v] == -CUDART_INF_F) ? 0.f : __expf(logit[v] - m);
    probs[tid * NQ + v] = e;
    float s = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) red_sum[v * 8 + warp] = s;
  }
  __syncthreads();

  // ---- P @ V: thread owns output columns c = tid, tid + 256, ... ----------
  const int nkeys = min(kAttnChunk, seq - chunk0);
  for (int c = tid; c < D; c += blockDim.x) {
    float o[NQ];
#pragma unroll
    for (int v = 0; v < NQ; ++v) o[v] = 0.f;
    for (int j = 0; j < nkeys; ++j) {
      const int kk = chunk0 + j;
      const int64_t blk = page_of(table, kk, p.block_size, p.max_blocks, p.num_blocks);
      if (blk < 0) continue;  // its probability is zero as well
      const uint8_t *row = p.vc + ((blk * p.block_size + kk % p.block_size) * p.kv_heads) * width + head_off;
      const float vs = *reinterpret_cast<const float *>(row + D);
      const float vv = bf16_bits_to_f32(f32_to_bf16_bits(lut[row[c]] * vs));
#pragma unroll
      for (int v = 0; v < NQ; ++v) o[v] = fmaf(probs[j * NQ + v], vv, o[v]);
    }
#pragma unroll
    for (int v = 0; v < NQ; ++v) {
      if (v >= nq) continue;
      float l = 0.f;
      for (int w = 0; w < 8; ++w) l += red_sum[v * 8 + w];
      const int r = v / group, gq = v - r * group;
      const int64_t tok = q0 + row_begin + r;
      const int64_t head = (int64_t)h * group + gq;
      if (p.splits == 1) {
        const float val = l > 0.f ? o[v] / l : 0.f;
        p.out[(tok * p.heads + head) * D + c] = (uint16_t)f32_to_bf16_bits(val);
      } else {
        float *dst = p.part + ((tok * p.heads + head) * p.splits + split) * part_stride(p.d);
        dst[c] = o[v];
        if (c == 0) {
          dst[D] = mx[v];
          dst[D + 1] = l;
        }
      }
    }
  }
}

// Merge the split partials of one (token, head): out = sum_s o_s e^(m_s - M)
// / sum_s l_s e^(m_s - M).  The split weights are computed once, in
// parallel, into shared memory (blocks of 1024 splits), then every thread
// sums its columns with independent loads.
constexpr int kCombineThreads = 256;
constexpr int kCombineBlock = 1024;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float *scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // scratch may still be read from a previous reduction
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = scratch[0];
  for (int w = 1; w < kCombineThreads / 32; ++w) v = is_max ? fmaxf(v, scratch[w]) : v + scratch[w];
  return v;
}

__global__ void __launch_bounds__(kCombineThreads) attention_combine_kernel(
    const float *__restrict__ part, int64_t rows, int64_t d, int splits, int chunk, const int32_t *q_start,
    const int32_t *seq_lens, int64_t batch, int64_t heads, uint16_t *__restrict__ out) {
  pdl_wait();  // inputs come from the previous kernel of the stream
  __shared__ float wgt[kCombineBlock];
  __shared__ float scratch[kCombineThreads / 32];
  const int64_t row = blockIdx.x;  // token * heads + head
  if (row >= rows) return;
  const int64_t tok = row / heads;
  // number of splits that hold keys for this token's request
  int64_t b = 0;
  while (b + 1 < batch && q_start[b + 1] <= tok) ++b;
  const int64_t need = ((int64_t)seq_lens[b] + chunk - 1) / chunk;
  const int used = (int)(need < splits ? need : splits);
  const int64_t stride = part_stride(d);
  const float *base = part + row * splits * stride;
  float M = -CUDART_INF_F;
  for (int s = threadIdx.x; s < used; s += kCombineThreads) M = fmaxf(M, base[s * stride + d]);
  M = block_reduce(M, true, scratch);
  float L = 0.f;
  for (int s = threadIdx.x; s < used; s += kCombineThreads) {
    const float ms = base[s * stride + d];
    if (ms != -CUDART_INF_F) L += base[s * stride + d + 1] * __expf(ms - M);
  }
  L = block_reduce(L, false, scratch);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // columns tid + 256 j (d <= 1024)
  for (int s0 = 0; s0 < used; s0 += kCombineBlock) {
    const int n = min(kCombineBlock, used - s0);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kCombineThreads) {
      const float ms = base[(s0 + i) * stride + d];
      wgt[i] = ms == -CUDART_INF_F ? 0.f : __expf(ms - M);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = threadIdx.x + (int64_t)kCombineThreads * j;
      if (c >= d) break;
      float a = acc[j];
      // unconditional loads (a split without keys has weight 0 and a zero
      // partial), so the unrolled splits' loads are in flight together
#pragma unroll 8
      for (int i = 0; i < n; ++i) a = fmaf(__ldg(base + (s0 + i) * stride + c), wgt[i], a);
      acc[j] = a;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t c = threadIdx.x + (int64_t)kCombineThreads * j;
    if (c < d) out[row * d + c] = (uint16_t)f32_to_bf16_bits(acc[j] * inv);
  }
}

// ------------------------------------------------------ decode attention ---

constexpr int kDecChunk = 64;   // keys per CTA of the decode kernel
constexpr int kDecThreads = 128;
constexpr int kDecHead = 256;   // head size of the decode kernel (128 threads x 2 value columns)
constexpr int kDecBatch = 8;    // key rows whose loads a warp issues together

// Split-KV attention for decode batches (normally one query row per
// request).  CTA = (request b, KV head h, 64-key chunk); the G query heads
// of the GQA group share every key and value load.
//   * the scales are static per head, so the CTA builds K and V tables of
//     BF16(decode(c) x scale) for the scale of its first row; a row with
//     that scale decodes with one lookup, any other row multiplies and
//     rounds as the reference materialises BF16 K and V;
//   * the chunk's row offsets are resolved from the block table once, into
//     shared memory (a block id outside [0, num_blocks) marks the key absent);
//   * scores: warp w takes keys w, w+4, ...; the 32 lanes read one K row
//     together (4 bytes per lane and 128-byte step, coalesced) and reduce the
//     G dot products with butterfly shuffles;
//   * softmax per head in FP32; P @ V with the same row split as the scores
//     (warp w takes keys [16 w, 16 w + 16)), the four warps' sums added in
//     shared memory; all row loads are unconditional, so the unrolled keys'
//     loads are in flight together;
//   * partials (unnormalised output, running max, sum) merge in
//     attention_combine_kernel, or are written directly when one chunk covers
//     the longest request.
template <int G>
__global__ void __launch_bounds__(kDecThreads) paged_decode_kernel(const AttnArgs p) {
  pdl_wait();  // inputs come from the previous kernel of the stream
  constexpr int D = kDecHead;
  constexpr int W = D / 128;  // 4-byte K / V words per lane per row
  __shared__ float lut[256], klut[256], vlut[256];
  __shared__ float ks0, vs0;
  __shared__ int64_t rowoff[kDecChunk];
  __shared__ float prob[G][kDecChunk];
  __shared__ float mrow[G], lrow[G];
  __shared__ __align__(16) float vsum[4][G][D];  // per-warp P @ V sums
  const int b = blockIdx.x / (int)p.kv_heads, h = blockIdx.x - b * (int)p.kv_heads;
  const int split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q0 = p.q_start[b], q_len = p.q_start[b + 1] - q0;
  const int seq = p.seq_lens[b];
  const int chunk0 = split * kDecChunk;
  if (q_len <= 0 || chunk0 >= seq) return;  // the merge reads only chunks that hold keys
  const int64_t width = D + 4;
  for (int i = tid; i < 256; i += kDecThreads) lut[i] = __uint_as_float(g_decode_f32.v[i]);
  if (tid < kDecChunk) {
    const int key = chunk0 + tid;
    int64_t off = -1;
    if (key < seq) {
      const int64_t blk = page_of(p.tables + (int64_t)b * p.max_blocks, key, p.block_size, p.max_blocks,
                                  p.num_blocks);
      if (blk >= 0) off = ((blk * p.block_size + key % p.block_size) * p.kv_heads + h) * width;
    }
    rowoff[tid] = off;
    if (tid == 0) {  // the chunk's reference scales (NaN: no table, every row computes)
      ks0 = off >= 0 ? *reinterpret_cast<const float *>(p.kc + off + D) : CUDART_NAN_F;
      vs0 = off >= 0 ? *reinterpret_cast<const float *>(p.vc + off + D) : CUDART_NAN_F;
    }
  }
  __syncthreads();
  for (int i = tid; i < 256; i += kDecThreads) {
    klut[i] = bf16_bits_to_f32(f32_to_bf16_bits(lut[i] * ks0));
    vlut[i] = bf16_bits_to_f32(f32_to_bf16_bits(lut[i] * vs0));
  }
  __syncthreads();

  for (int r = 0; r < q_len; ++r) {
    const int64_t tok = q0 + r;
    const int limit = p.causal ? seq - q_len + r : seq - 1;  // last key this row sees
    // query vectors: lane holds columns 4 (lane + 32 i) + e of every head g
    float qv[G][4 * W];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint16_t *qrow = p.q + (tok * p.heads + (int64_t)h * G + g) * D;
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const uint2 v = *reinterpret_cast<const uint2 *>(qrow + 4 * (lane + 32 * i));
        qv[g][4 * i + 0] = bf16_bits_to_f32(v.x & 0xFFFFu);
        qv[g][4 * i + 1] = bf16_bits_to_f32(v.x >> 16);
        qv[g][4 * i + 2] = bf16_bits_to_f32(v.y & 0xFFFFu);
        qv[g][4 * i + 3] = bf16_bits_to_f32(v.y >> 16);
      }
    }
    // ---- scores, kKB = 32 / G keys per batch: all the batch's row loads
    // (read-only path, unconditional: an absent key reads row 0 of the cache,
    // in bounds, and is masked afterwards) are issued before any arithmetic
    // or shared-memory store, so they are in flight together.  The batch's
    // 32 (key, head) partial dot products are then summed across the warp by
    // a transpose-reduction: after 16 + 8 + 4 + 2 + 1 shuffles lane l holds
    // the total of value l.
    constexpr int kKB = 32 / G < kDecChunk / 4 ? 32 / G : kDecChunk / 4;
    for (int j0 = 0; j0 < kDecChunk / 4; j0 += kKB) {
      uint32_t kw[kKB][W];
      float ks[kKB];
#pragma unroll
      for (int u = 0; u < kKB; ++u) {
        const int k = warp + 4 * (j0 + u);
        const int64_t off = rowoff[k];
        const uint8_t *row = p.kc + (off >= 0 ? off : 0);
        ks[u] = __ldg(reinterpret_cast<const float *>(row + D));
#pragma unroll
        for (int i = 0; i < W; ++i) kw[u][i] = __ldg(reinterpret_cast<const unsigned int *>(row + 4 * (lane + 32 * i)));
      }
      float part[32];  // value u * G + g: key j0 + u, head g (unused values stay 0)
#pragma unroll
      for (int i = kKB * G; i < 32; ++i) part[i] = 0.f;
#pragma unroll
      for (int u = 0; u < kKB; ++u) {
#pragma unroll
        for (int g = 0; g < G; ++g) part[u * G + g] = 0.f;
        if (ks[u] == ks0) {  // uniform across the warp
#pragma unroll
          for (int i = 0; i < W; ++i) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float kv = klut[(kw[u][i] >> (8 * e)) & 0xFFu];
#pragma unroll
              for (int g = 0; g < G; ++g) part[u * G + g] = fmaf(qv[g][4 * i + e], kv, part[u * G + g]);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < W; ++i) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float kv = bf16_bits_to_f32(f32_to_bf16_bits(lut[(kw[u][i] >> (8 * e)) & 0xFFu] * ks[u]));
#pragma unroll
              for (int g = 0; g < G; ++g) part[u * G + g] = fmaf(qv[g][4 * i + e], kv, part[u * G + g]);
            }
          }
        }
      }
#pragma unroll
      for (int half = 16; half > 0; half >>= 1) {
        const bool upper = (lane & half) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? part[i] : part[i + half];
          const float keep = upper ? part[i + half] : part[i];
          part[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, half);
        }
      }
      // lane l = u * G + g now holds the score of key j0 + u, head g
      {
        const int u = lane / G, g = lane - u * G;
        if (u < kKB) {
          const int k = warp + 4 * (j0 + u);
          const bool valid = rowoff[k] >= 0 && chunk0 + k <= limit;
          prob[g][k] = valid ? part[0] * p.scale : -CUDART_INF_F;
        }
      }
    }
    __syncthreads();
    // ---- softmax per head (warp w takes heads w, w + 4)
    for (int g = warp; g < G; g += 4) {
      float v[kDecChunk / 32];
      float m = -CUDART_INF_F;
#pragma unroll
      for (int i = 0; i < kDecChunk / 32; ++i) {
        v[i] = prob[g][lane + 32 * i];
        m = fmaxf(m, v[i]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
      float l = 0.f;
#pragma unroll
      for (int i = 0; i < kDecChunk / 32; ++i) {
        const float e = v[i] == -CUDART_INF_F ? 0.f : __expf(v[i] - m);
        prob[g][lane + 32 * i] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
      if (lane == 0) {
        mrow[g] = m;
        lrow[g] = l;
      }
    }
    __syncthreads();
    // ---- P @ V: warp w takes keys [32 w, 32 w + 32) and, like the K pass,
    // lane columns 4 (lane + 32 i) + e; the four warps' sums meet in shared
    // memory afterwards
    float acc[G][4 * W];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int c = 0; c < 4 * W; ++c) acc[g][c] = 0.f;
    constexpr int kKeysPerWarp = kDecChunk / 4;
    for (int j0 = 0; j0 < kKeysPerWarp; j0 += kDecBatch) {
      uint32_t vw[kDecBatch][W];
      float vs[kDecBatch];
      bool valid[kDecBatch];
#pragma unroll
      for (int u = 0; u < kDecBatch; ++u) {
        const int k = warp * kKeysPerWarp + j0 + u;
        const int64_t off = rowoff[k];
        valid[u] = off >= 0 && chunk0 + k <= limit;
        const uint8_t *row = p.vc + (valid[u] ? off : 0);
        vs[u] = __ldg(reinterpret_cast<const float *>(row + D));
#pragma unroll
        for (int i = 0; i < W; ++i) vw[u][i] = __ldg(reinterpret_cast<const unsigned int *>(row + 4 * (lane + 32 * i)));
      }
#pragma unroll
      for (int u = 0; u < kDecBatch; ++u) {
        if (!valid[u]) continue;
        const int k = warp * kKeysPerWarp + j0 + u;
        float pk[G];
#pragma unroll
        for (int g = 0; g < G; ++g) pk[g] = prob[g][k];
        const bool table = vs[u] == vs0;
#pragma unroll
        for (int i = 0; i < W; ++i) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t c = (vw[u][i] >> (8 * e)) & 0xFFu;
            const float vv = table ? vlut[c] : bf16_bits_to_f32(f32_to_bf16_bits(lut[c] * vs[u]));
#pragma unroll
            for (int g = 0; g < G; ++g) acc[g][4 * i + e] = fmaf(pk[g], vv, acc[g][4 * i + e]);
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < W; ++i)
        *reinterpret_cast<float4 *>(&vsum[warp][g][4 * (lane + 32 * i)]) =
            make_float4(acc[g][4 * i], acc[g][4 * i + 1], acc[g][4 * i + 2], acc[g][4 * i + 3]);
    __syncthreads();
    // thread t finishes columns 2 t and 2 t + 1 of every head
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        o0 += vsum[w][g][2 * tid];
        o1 += vsum[w][g][2 * tid + 1];
      }
      const int64_t head = (int64_t)h * G + g;
      if (p.splits == 1) {
        const float l = lrow[g];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint16_t *dst = p.out + (tok * p.heads + head) * D;
        *reinterpret_cast<uint32_t *>(dst + 2 * tid) = f32_to_bf16_bits(o0 * inv) | (f32_to_bf16_bits(o1 * inv) << 16);
      } else {
        float *dst = p.part + ((tok * p.heads + head) * p.splits + split) * part_stride(D);
        dst[2 * tid] = o0;
        dst[2 * tid + 1] = o1;
        if (tid == 0) {
          dst[D] = mrow[g];
          dst[D + 1] = lrow[g];
        }
      }
    }
    __syncthreads();  // prob / mrow / lrow are reused by the next query row
  }
}

// ------------------------------------------------------- gather decode ---

__global__ void __launch_bounds__(256) kv_gather_decode_kernel(const uint8_t *__restrict__ cache,
                                                               const int32_t *__restrict__ tables,
                                                               const int32_t *__restrict__ seq_lens,
                                                               const int32_t *__restrict__ out_start, int64_t batch,
                                                               int64_t heads, int64_t d, int64_t block_size,
                                                               int64_t max_blocks, int64_t num_blocks,
                                                               int64_t max_seq, uint16_t *__restrict__ out) {
  __shared__ float lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = __uint_as_float(g_decode_f32.v[i]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t width = d + 4;
  const int64_t total = batch * max_seq * heads;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < total;
       row += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t b = row / (max_seq * heads);
    const int64_t rem = row - b * max_seq * heads;
    const int64_t i = rem / heads, h = rem - i * heads;
    if (i >= seq_lens[b]) continue;
    const int64_t blk = page_of(tables + b * max_blocks, i, block_size, max_blocks, num_blocks);
    uint16_t *dst = out + ((out_start[b] + i) * heads + h) * d;
    if (blk < 0) {  // uncovered position: zeros, like an unwritten page row
      for (int64_t c = lane * 4; c < d; c += 128) *reinterpret_cast<uint2 *>(dst + c) = make_uint2(0, 0);
      continue;
    }
    const uint8_t *src = cache + ((blk * block_size + i % block_size) * heads + h) * width;
    const float s = *reinterpret_cast<const float *>(src + d);
    for (int64_t c = lane * 4; c < d; c += 128) {
      const uint32_t w = *reinterpret_cast<const uint32_t *>(src + c);
      uint2 o;
      o.x = f32_to_bf16_bits(lut[w & 0xFFu] * s) | (f32_to_bf16_bits(lut[(w >> 8) & 0xFFu] * s) << 16);
      o.y = f32_to_bf16_bits(lut[(w >> 16) & 0xFFu] * s) | (f32_to_bf16_bits(lut[w >> 24] * s) << 16);
      *reinterpret_cast<uint2 *>(dst + c) = o;
    }
  }
}

static int attn_grid_cap(int64_t work) {
  const int64_t cap = (int64_t)num_sms() * 8;
  return (int)(work < cap ? (work > 0 ? work : 1) : cap);
}

}  // namespace hif8

using namespace hif8;

extern "C" int hif8_kv_cache_write(const void *key, const void *value, int src_dtype, int64_t tokens,
                                   int64_t kv_heads, int64_t head_size, int64_t src_token_stride,
                                   const float *key_scale, const float *value_scale,
                                   const int64_t *slot_mapping, uint8_t *key_cache, uint8_t *value_cache,
                                   int64_t num_blocks, int64_t block_size, int32_t *bad_slots, void *stream) {
  if (tokens < 0 || kv_heads <= 0 || head_size <= 0 || head_size % 4 != 0 || num_blocks <= 0 ||
      block_size <= 0 || src_token_stride < kv_heads * head_size || src_token_stride % 4 != 0)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (src_dtype != HIF8_DTYPE_F16 && src_dtype != HIF8_DTYPE_BF16) return HIF8_ERR_INVALID_ARGUMENT;
  if (!key || !key_scale || !key_cache || (tokens > 0 && !slot_mapping)) return HIF8_ERR_INVALID_ARGUMENT;
  // 8-byte source loads and 4-byte page stores
  if ((reinterpret_cast<uintptr_t>(key) & 7u) || (value && (reinterpret_cast<uintptr_t>(value) & 7u)) ||
      (reinterpret_cast<uintptr_t>(key_cache) & 3u) || (value_cache && (reinterpret_cast<uintptr_t>(value_cache) & 3u)))
    return HIF8_ERR_INVALID_ARGUMENT;
  const bool with_v = value != nullptr;
  if (with_v && (!value_scale || !value_cache)) return HIF8_ERR_INVALID_ARGUMENT;
  if (tokens == 0) return HIF8_OK;
  KvWriteArgs p{};
  p.src[0] = static_cast<const uint16_t *>(key);
  p.src[1] = static_cast<const uint16_t *>(value);
  p.scale[0] = key_scale;
  p.scale[1] = value_scale;
  p.cache[0] = key_cache;
  p.cache[1] = value_cache;
  p.slots = slot_mapping;
  p.bad_slots = bad_slots;
  p.tokens = tokens;
  p.heads = kv_heads;
  p.d = head_size;
  p.token_stride = src_token_stride;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.planes = with_v ? 2 : 1;
  const int64_t warps = tokens * kv_heads * p.planes;
  const int grid = attn_grid_cap((warps + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return src_dtype == HIF8_DTYPE_BF16 ? launch_pdl(kv_write_kernel<HIF8_DTYPE_BF16>, dim3(grid), dim3(256), 0, s, p)
                                      : launch_pdl(kv_write_kernel<HIF8_DTYPE_F16>, dim3(grid), dim3(256), 0, s, p);
}

static int attn_nq(int64_t group, int64_t q_rows) { return (int)(group * q_rows); }

// Sized for the finer of the two kernels' key chunks (the decode kernel's).
extern "C" size_t hif8_paged_attention_workspace_size(int64_t num_tokens, int64_t num_heads, int64_t head_size,
                                                      int64_t max_seq_len) {
  const int64_t splits = (max_seq_len + kDecChunk - 1) / kDecChunk;
  if (splits <= 1) return 0;
  return (size_t)(num_tokens * num_heads * splits * part_stride(head_size)) * sizeof(float);
}

template <int NQ>
static int launch_attention(AttnArgs p, int64_t batch, int64_t q_groups, cudaStream_t s) {
  const size_t smem = (256 + (size_t)NQ * p.d + (size_t)kAttnChunk * NQ + 2 * NQ * 8) * sizeof(float);
  auto kernel = paged_attention_kernel<NQ>;
  const int st = ensure_smem_limit(reinterpret_cast<const void *>(kernel), smem);
  if (st != HIF8_OK) return st;
  dim3 grid((unsigned)(batch * p.kv_heads), (unsigned)p.splits, (unsigned)q_groups);
  kernel<<<grid, kAttnThreads, smem, s>>>(p);
  return check_launch();
}

extern "C" int hif8_paged_attention(const uint16_t *query, const uint8_t *key_cache, const uint8_t *value_cache,
                                    const int32_t *block_tables, const int32_t *seq_lens,
                                    const int32_t *query_start, int64_t batch, int64_t num_tokens,
                                    int64_t num_heads, int64_t kv_heads, int64_t head_size, int64_t num_blocks,
                                    int64_t block_size, int64_t max_blocks, int64_t max_seq_len,
                                    float softmax_scale, int causal,
                                    uint16_t *out, void *workspace, size_t workspace_bytes, void *stream) {
  if (batch <= 0 || num_tokens < 0 || num_heads <= 0 || kv_heads <= 0 || num_heads % kv_heads != 0 ||
      head_size <= 0 || head_size % 4 != 0 || head_size > 1024 || num_blocks <= 0 || block_size <= 0 ||
      max_blocks <= 0 || max_seq_len < 0)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (!query || !key_cache || !value_cache || !block_tables || !seq_lens || !query_start || !out)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return HIF8_OK;
  const int64_t group = num_heads / kv_heads;
  if (group > 16) return HIF8_ERR_INVALID_ARGUMENT;
  const size_t need = hif8_paged_attention_workspace_size(num_tokens, num_heads, head_size, max_seq_len);
  if (need > 0 && (!workspace || workspace_bytes < need)) return HIF8_ERR_WORKSPACE;
  // decode batches (as many query rows as requests) of head size 256 and a
  // power-of-two GQA group take the split-KV decode kernel
  const bool decode = num_tokens == batch && head_size == kDecHead &&
                      (group == 1 || group == 2 || group == 4 || group == 8) &&
                      (reinterpret_cast<uintptr_t>(query) & 7u) == 0 && (reinterpret_cast<uintptr_t>(out) & 3u) == 0;
  const int chunk = decode ? kDecChunk : kAttnChunk;
  const int64_t splits = max_seq_len > 0 ? (max_seq_len + chunk - 1) / chunk : 1;
  AttnArgs p{};
  p.q = query;
  p.kc = key_cache;
  p.vc = value_cache;
  p.tables = block_tables;
  p.seq_lens = seq_lens;
  p.q_start = query_start;
  p.out = out;
  p.part = static_cast<float *>(workspace);
  p.heads = num_heads;
  p.kv_heads = kv_heads;
  p.d = head_size;
  p.block_size = block_size;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.splits = (int)splits;
  p.scale = softmax_scale;
  p.causal = causal;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // query rows per CTA: every query vector of a CTA shares the key loads
  int status;
  if (decode) {
    const dim3 grid((unsigned)(batch * kv_heads), (unsigned)splits, 1);
    switch (group) {
      case 1: status = launch_pdl(paged_decode_kernel<1>, grid, dim3(kDecThreads), 0, s, p); break;
      case 2: status = launch_pdl(paged_decode_kernel<2>, grid, dim3(kDecThreads), 0, s, p); break;
      case 4: status = launch_pdl(paged_decode_kernel<4>, grid, dim3(kDecThreads), 0, s, p); break;
      default: status = launch_pdl(paged_decode_kernel<8>, grid, dim3(kDecThreads), 0, s, p); break;
    }
  } else if (group <= 4) {
    // prefill and mixed batches: up to 4 query vectors per CTA
    p.q_rows_per_cta = (int)(4 / group);
    const int64_t q_groups = (num_tokens + p.q_rows_per_cta - 1) / p.q_rows_per_cta;
    status = launch_attention<4>(p, batch, q_groups, s);
  } else {
    p.q_rows_per_cta = (int)(16 / group);
    const int64_t q_groups = (num_tokens + p.q_rows_per_cta - 1) / p.q_rows_per_cta;
    status = launch_attention<16>(p, batch, q_groups, s);
  }
  (void)attn_nq;
  if (status != HIF8_OK || splits == 1) return status;
  const int64_t rows = num_tokens * num_heads;
  return launch_pdl(attention_combine_kernel, dim3((unsigned)rows), dim3(kCombineThreads), 0, s, (const float *)p.part,
                    rows, head_size, (int)splits, chunk, query_start, seq_lens, batch, num_heads, out);
}

extern "C" int hif8_kv_gather_decode(const uint8_t *cache, const int32_t *block_tables, const int32_t *seq_lens,
                                     const int32_t *out_start, int64_t batch, int64_t kv_heads, int64_t head_size,
                                     int64_t num_blocks, int64_t block_size, int64_t max_blocks,
                                     int64_t max_seq_len, uint16_t *out, void *stream) {
  if (batch <= 0 || kv_heads <= 0 || head_size <= 0 || head_size % 4 != 0 || num_blocks <= 0 || block_size <= 0 ||
      max_blocks <= 0 || max_seq_len < 0)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (!cache || !block_tables || !seq_lens || !out_start || !out) return HIF8_ERR_INVALID_ARGUMENT;
  if (max_seq_len == 0) return HIF8_OK;
  const int64_t warps = batch * max_seq_len * kv_heads;
  kv_gather_decode_kernel<<<attn_grid_cap((warps + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      cache, block_tables, seq_lens, out_start, batch, kv_heads, head_size, block_size, max_blocks, num_blocks,
      max_seq_len, out);
  return check_launch();
}
