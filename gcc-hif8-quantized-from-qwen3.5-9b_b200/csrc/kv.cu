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
// / sum_s l_s e^(m_s - M).
__global__ void __launch_bounds__(256) attention_combine_kernel(const float *__restrict__ part, int64_t rows,
                                                                int64_t d, int splits, const int32_t *q_start,
                                                                const int32_t *seq_lens, int64_t batch,
                                                                int64_t heads, uint16_t *__restrict__ out) {
  const int64_t row = blockIdx.x;  // token * heads + head
  if (row >= rows) return;
  const int64_t tok = row / heads;
  // number of splits that hold keys for this token's request
  int64_t b = 0;
  while (b + 1 < batch && q_start[b + 1] <= tok) ++b;
  const int64_t need = ((int64_t)seq_lens[b] + kAttnChunk - 1) / kAttnChunk;
  const int used = (int)(need < splits ? need : splits);
  const float *base = part + row * splits * part_stride(d);
  float M = -CUDART_INF_F;
  for (int s = 0; s < used; ++s) M = fmaxf(M, base[s * part_stride(d) + d]);
  float L = 0.f;
  for (int s = 0; s < used; ++s) {
    const float ms = base[s * part_stride(d) + d];
    if (ms != -CUDART_INF_F) L += base[s * part_stride(d) + d + 1] * __expf(ms - M);
  }
  for (int64_t c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < used; ++s) {
      const float ms = base[s * part_stride(d) + d];
      if (ms != -CUDART_INF_F) acc += base[s * part_stride(d) + c] * __expf(ms - M);
    }
    out[row * d + c] = (uint16_t)f32_to_bf16_bits(L > 0.f ? acc / L : 0.f);
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
  if (src_dtype == HIF8_DTYPE_BF16) kv_write_kernel<HIF8_DTYPE_BF16><<<grid, 256, 0, s>>>(p);
  else kv_write_kernel<HIF8_DTYPE_F16><<<grid, 256, 0, s>>>(p);
  return check_launch();
}

static int attn_nq(int64_t group, int64_t q_rows) { return (int)(group * q_rows); }

extern "C" size_t hif8_paged_attention_workspace_size(int64_t num_tokens, int64_t num_heads, int64_t head_size,
                                                      int64_t max_seq_len) {
  const int64_t splits = (max_seq_len + kAttnChunk - 1) / kAttnChunk;
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
  const int64_t splits = max_seq_len > 0 ? (max_seq_len + kAttnChunk - 1) / kAttnChunk : 1;
  const size_t need = hif8_paged_attention_workspace_size(num_tokens, num_heads, head_size, max_seq_len);
  if (need > 0 && (!workspace || workspace_bytes < need)) return HIF8_ERR_WORKSPACE;
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
  if (group <= 4) {
    // decode steps (one query row per request) take the small variant
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
  attention_combine_kernel<<<(unsigned)rows, 256, 0, s>>>(p.part, rows, head_size, (int)splits, query_start,
                                                         seq_lens, batch, num_heads, out);
  return check_launch();
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
