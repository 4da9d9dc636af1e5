// Paged HiF8 KV cache: fused static write, paged attention that decodes only
// the touched pages, and the dense gather-decode of kv_runtime._gather_dense_hif8.
//
// Page layout (reference src/vllm_ascend_hif8/kv_cache.py:26-88): a cache is
// [num_blocks, block_size, kv_heads, head_size + 4] bytes; each row holds
// head_size HiF8 codes followed by the row's little-endian FP32 scale.
// Consecutive blocks of a cache may sit further apart than one block's
// bytes (block_stride): vLLM's block-major page holds a block's K rows and
// then its V rows, so each plane's blocks are two block images apart.
#include <math_constants.h>

#include <atomic>
#include <type_traits>

#include "hif8_common.cuh"

namespace hif8 {

// ------------------------------------------------------------ KV write ---

// Static quantisation of one K/V element with its head's scale: the rule of
// hif8_static_quant (static_code), so page bytes equal the quantised rows.
__device__ __forceinline__ uint32_t kv_quant_one(float f, float r, double r64, bool exact_only,
                                                 const uint8_t *__restrict__ tbl) {
  return static_code(f, r, r64, exact_only, tbl);
}

struct KvWriteArgs {
  const uint16_t *src[2];  // key, value: [tokens, heads, D] with token stride
  const float *scale[2];   // per head
  uint8_t *cache[2];
  const int64_t *slots;
  int32_t *bad_slots;
  int64_t tokens, heads, d, token_stride, num_blocks, block_size;
  int64_t block_stride;  // bytes between consecutive blocks of a cache
  int64_t cache_slots;  // num_blocks * block_size: slots at or above are out of range
  int64_t units;        // planes * tokens * heads * (d / elements per unit), < 2^32
  int planes;           // 1 = K only, 2 = K and V
};

// Byte offset of the row group (every head's row) of slot `slot` in a
// cache: slot * group for dense blocks, otherwise block * block_stride +
// offset * group (one division, once per row group).
__device__ __forceinline__ int64_t kv_slot_offset(const KvWriteArgs &p, int64_t slot, int64_t group) {
  if (p.block_stride == p.block_size * group) return slot * group;
  const int64_t blk = slot / p.block_size;
  return blk * p.block_stride + (slot - blk * p.block_size) * group;
}

constexpr int kKvUnroll = 4;      // units in flight per thread
constexpr int kKvScaleSlots = 64;  // heads whose scale / reciprocal a CTA stages in shared memory

// Quantise ELEMS consecutive elements of one (plane, token, head) row per
// unit (ELEMS = 16: two 16-byte loads; 4: one 8-byte load) and store them
// into the row's page slot with 4-byte stores (a page row is D + 4 bytes,
// so rows are only 4-byte aligned).  A page row starts at
// (slot * heads + head) * (D + 4) in dense blocks (slot = block * block_size
// + offset, so no division is needed; kv_slot_offset otherwise); a slot at
// or beyond num_blocks * block_size is out of range (counted once per
// token), a negative slot is skipped.  The unit
// holding a row's last elements also writes the row's FP32 scale.  Every
// thread keeps kKvUnroll units in flight (slot and source loads of all of
// them first), and the per-head reciprocals are formed once per CTA.
template <int kDtype, int ELEMS>
__global__ void __launch_bounds__(256) kv_write_kernel(const KvWriteArgs p) {
  __shared__ __align__(16) uint8_t tbl[4096];
  __shared__ float sh_s[2 * kKvScaleSlots], sh_r[2 * kKvScaleSlots];
  __shared__ double sh_r64[2 * kKvScaleSlots];
  __shared__ uint8_t sh_exact[2 * kKvScaleSlots];
  load_encode_mag_table(tbl);  // module data: before the dependency wait
  pdl_wait();  // inputs come from the previous kernel of the stream
  const bool staged = p.heads <= kKvScaleSlots;
  if (staged) {
    for (int i = threadIdx.x; i < p.planes * p.heads; i += blockDim.x) {
      const int plane = i / (int)p.heads, h = i - plane * (int)p.heads;
      const float s = p.scale[plane][h];
      const float r = __frcp_rn(s);
      const uint32_t re = __float_as_uint(r) & 0x7F800000u;
      sh_s[plane * kKvScaleSlots + h] = s;
      sh_r[plane * kKvScaleSlots + h] = r;
      sh_r64[plane * kKvScaleSlots + h] = __drcp_rn((double)s);
      sh_exact[plane * kKvScaleSlots + h] = (re == 0u) | (re == 0x7F800000u) | !(s > 0.f);
    }
  }
  __syncthreads();
  const uint32_t upr = (uint32_t)(p.d / ELEMS);  // units per row
  const uint32_t heads = (uint32_t)p.heads;
  const uint32_t per_plane = (uint32_t)(p.units / p.planes);
  const int64_t width = p.d + 4;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t u0 = blockIdx.x * blockDim.x + threadIdx.x; u0 < (uint32_t)p.units; u0 += kKvUnroll * stride) {
    int64_t slot[kKvUnroll];
    uint32_t row[kKvUnroll], chunk[kKvUnroll];
    int plane[kKvUnroll];
    uint4 a[kKvUnroll], b[kKvUnroll];
#pragma unroll
    for (int u = 0; u < kKvUnroll; ++u) {
      const uint64_t uu = (uint64_t)u0 + (uint64_t)u * stride;
      slot[u] = -1;
      if (uu < (uint64_t)p.units) {
        plane[u] = uu >= per_plane;
        const uint32_t rem = (uint32_t)uu - (plane[u] ? per_plane : 0u);
        row[u] = rem / upr;
        chunk[u] = rem - row[u] * upr;
        const uint32_t tok = row[u] / heads;
        slot[u] = __ldg(p.slots + tok);
        const uint16_t *src = p.src[plane[u]] + (int64_t)tok * p.token_stride +
                              (int64_t)(row[u] - tok * heads) * p.d + (int64_t)chunk[u] * ELEMS;
        if constexpr (ELEMS == 16) {
          a[u] = __ldcs(reinterpret_cast<const uint4 *>(src));
          b[u] = __ldcs(reinterpret_cast<const uint4 *>(src) + 1);
        } else {
          const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(src));
          a[u] = make_uint4(v.x, v.y, 0, 0);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kKvUnroll; ++u) {
      if (slot[u] < 0) continue;  // skipped (negative) or past the end of the work
      const uint32_t tok = row[u] / heads, h = row[u] - tok * heads;
      if (slot[u] >= p.cache_slots) {
        if (p.bad_slots && plane[u] == 0 && h == 0 && chunk[u] == 0) atomicAdd(p.bad_slots, 1);
        continue;
      }
      float s, r;
      double r64;
      bool exact_only;
      if (staged) {
        s = sh_s[plane[u] * kKvScaleSlots + h];
        r = sh_r[plane[u] * kKvScaleSlots + h];
        r64 = sh_r64[plane[u] * kKvScaleSlots + h];
        exact_only = sh_exact[plane[u] * kKvScaleSlots + h] != 0;
      } else {
        s = p.scale[plane[u]][h];
        r = __frcp_rn(s);
        r64 = __drcp_rn((double)s);
        const uint32_t re = __float_as_uint(r) & 0x7F800000u;
        exact_only = (re == 0u) | (re == 0x7F800000u) | !(s > 0.f);
      }
      uint8_t *dst_row = p.cache[plane[u]] + kv_slot_offset(p, slot[u], (int64_t)heads * width) + h * width;
      uint32_t *dst = reinterpret_cast<uint32_t *>(dst_row + (int64_t)chunk[u] * ELEMS);
      const uint32_t w[8] = {a[u].x, a[u].y, a[u].z, a[u].w, b[u].x, b[u].y, b[u].z, b[u].w};
      uint32_t o[4];
      // the 16-element chunk path (one check per chunk); each element by
      // division-capable static_code where that check fails
      if constexpr (ELEMS == 16) {
        if (exact_only || !scale_edge_ok(s) || !static_codes16<kDtype>(w, s, r, 0.5f * s, tbl, o))
          static_codes16_exact<kDtype>(w, r64, tbl, o);
      } else {
        const uint32_t lo = w[0], hi = w[1];
        const uint32_t b0 = kv_quant_one(half_bits_to_f32<kDtype>(lo & 0xFFFFu), r, r64, exact_only, tbl);
        const uint32_t b1 = kv_quant_one(half_bits_to_f32<kDtype>(lo >> 16), r, r64, exact_only, tbl);
        const uint32_t b2 = kv_quant_one(half_bits_to_f32<kDtype>(hi & 0xFFFFu), r, r64, exact_only, tbl);
        const uint32_t b3 = kv_quant_one(half_bits_to_f32<kDtype>(hi >> 16), r, r64, exact_only, tbl);
        o[0] = __byte_perm(b0 | (b1 << 8), b2 | (b3 << 8), 0x5410u);
      }
#pragma unroll
      for (int j = 0; j < ELEMS / 4; ++j) dst[j] = o[j];
      if (chunk[u] == upr - 1) *reinterpret_cast<float *>(dst_row + p.d) = s;
    }
  }
}

// One warp per (plane, token): the token's heads x D source elements (one
// contiguous run: head rows are D apart inside a token) are quantised into a
// shared-memory image of the token's page row group -- heads rows of D codes
// and the FP32 scale, (D + 4) bytes apart -- and the warp then writes the
// group (kv_slot_offset: slot * heads * (D + 4) bytes into dense blocks) with consecutive
// lanes on consecutive 16-byte words (4-byte words when the group size or
// base is not a multiple of 16): full, coalesced sectors instead of four
// 4-byte stores per 16 codes 16 bytes apart.  Chunk c (16 elements) of the
// token is head c >> kv_shift, offset (c & (D/16 - 1)) * 16: D / 16 is a
// power of two, so no division.  Scales that are powers of two take the
// check-free encode.  kKvWarpKeep chunks per lane are loaded before any is
// encoded.
constexpr int kKvWarps = 8;      // warps per CTA
constexpr int kKvWarpKeep = 2;   // 16-element chunks per lane in flight
constexpr int kKvGroupMax = 8192;  // largest row group (heads * (D + 4) bytes) staged per warp

struct KvWarpArgs {
  KvWriteArgs p;
  int shift;           // log2(D / 16)
  int group;           // heads * (D + 4) bytes
  int group_stage;     // group rounded up to 16 bytes (per-warp stage stride)
  int store16;         // the groups of both caches start on 16-byte boundaries
};

template <int kDtype>
__global__ void __launch_bounds__(kKvWarps * 32, 3) kv_write_warp_kernel(const KvWarpArgs a) {
  extern __shared__ __align__(16) uint8_t kv_smem[];
  uint8_t *tbl = kv_smem;                                  // 4 KB encode table
  float *sh_s = reinterpret_cast<float *>(kv_smem + 4096);  // [2][kKvScaleSlots]
  float *sh_r = sh_s + 2 * kKvScaleSlots;
  uint32_t *sh_mode = reinterpret_cast<uint32_t *>(sh_r + 2 * kKvScaleSlots);  // 0 check, 1 pow2, 2 exact only
  double *sh_r64 = reinterpret_cast<double *>(sh_mode + 2 * kKvScaleSlots);
  uint8_t *stage_all = reinterpret_cast<uint8_t *>(sh_r64 + 2 * kKvScaleSlots);
  const KvWriteArgs &p = a.p;
  load_encode_mag_table(tbl);  // module data: before the dependency wait
  pdl_wait();                  // inputs come from the previous kernel of the stream
  for (int i = threadIdx.x; i < p.planes * p.heads; i += blockDim.x) {
    const int plane = i / (int)p.heads, h = i - plane * (int)p.heads;
    const float sc = p.scale[plane][h];
    bool exact_only, pow2;
    double r64;
    const float r = __frcp_rn(sc);
    const uint32_t re = __float_as_uint(r) & 0x7F800000u;
    exact_only = (re == 0u) | (re == 0x7F800000u) | !(sc > 0.f);
    pow2 = scale_is_pow2(sc);
    r64 = __drcp_rn((double)sc);
    sh_s[plane * kKvScaleSlots + h] = sc;
    sh_r[plane * kKvScaleSlots + h] = r;
    sh_r64[plane * kKvScaleSlots + h] = r64;
    // 0: quotient from the product, 1: power of two, 2: exact FP64 path
    sh_mode[plane * kKvScaleSlots + h] = exact_only || !scale_edge_ok(sc) ? 2u : (pow2 ? 1u : 0u);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t *stage = stage_all + warp * a.group_stage;
  const int d = (int)p.d, width = d + 4;
  const int nchunks = (int)p.heads << a.shift;  // 16-element chunks per token
  const int64_t items = (int64_t)p.planes * p.tokens;
  for (int64_t it = (int64_t)blockIdx.x * kKvWarps + warp; it < items; it += (int64_t)gridDim.x * kKvWarps) {
    const int plane = it >= p.tokens;
    const int64_t tok = it - (plane ? p.tokens : 0);
    const int64_t slot = __ldg(p.slots + tok);  // warp-uniform
    const uint4 *src = reinterpret_cast<const uint4 *>(p.src[plane] + tok * p.token_stride);
    // the first source loads go out with the slot load (they do not depend
    // on it), so the two latencies overlap
    uint4 va[kKvWarpKeep], vb[kKvWarpKeep];
#pragma unroll
    for (int u = 0; u < kKvWarpKeep; ++u) {
      const int c = u * 32 + lane;
      if (c < nchunks) {
        va[u] = __ldcs(src + 2 * c);
        vb[u] = __ldcs(src + 2 * c + 1);
      }
    }
    if (slot < 0) continue;
    if (slot >= p.cache_slots) {
      if (p.bad_slots && plane == 0 && lane == 0) atomicAdd(p.bad_slots, 1);
      continue;
    }
    for (int c0 = 0; c0 < nchunks; c0 += 32 * kKvWarpKeep) {
      if (c0 > 0) {
#pragma unroll
        for (int u = 0; u < kKvWarpKeep; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < nchunks) {
            va[u] = __ldcs(src + 2 * c);
            vb[u] = __ldcs(src + 2 * c + 1);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kKvWarpKeep; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= nchunks) break;
        const int h = c >> a.shift;
        const int slot_h = plane * kKvScaleSlots + h;
        const float r = sh_r[slot_h];
        const uint32_t mode = sh_mode[slot_h];
        const uint32_t w[8] = {va[u].x, va[u].y, va[u].z, va[u].w, vb[u].x, vb[u].y, vb[u].z, vb[u].w};
        uint32_t o[4];
        if (mode == 1u) {
          static_codes16_pow2<kDtype>(w, r, tbl, o);
        } else if (mode == 2u ||
                   !static_codes16<kDtype>(w, sh_s[slot_h], r, 0.5f * sh_s[slot_h], tbl, o)) {
          static_codes16_exact<kDtype>(w, sh_r64[slot_h], tbl, o);
        }
        uint32_t *dst = reinterpret_cast<uint32_t *>(stage + h * width + ((c & ((1 << a.shift) - 1)) << 4));
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = o[j];
      }
    }
    for (int h = lane; h < (int)p.heads; h += 32)
      *reinterpret_cast<float *>(stage + h * width + d) = sh_s[plane * kKvScaleSlots + h];
    __syncwarp();
    uint8_t *dst = p.cache[plane] + kv_slot_offset(p, slot, a.group);
    if (a.store16) {
      for (int i = lane; i < (a.group >> 4); i += 32)
        __stcs(reinterpret_cast<uint4 *>(dst) + i, reinterpret_cast<const uint4 *>(stage)[i]);
    } else {
      for (int i = lane; i < (a.group >> 2); i += 32)
        __stcs(reinterpret_cast<uint32_t *>(dst) + i, reinterpret_cast<const uint32_t *>(stage)[i]);
    }
    __syncwarp();  // the stage is rewritten by the warp's next token
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
  int64_t block_stride;       // bytes between consecutive blocks of a cache
  int splits;                 // KV chunks per request (grid.y)
  int chunk;                  // keys per chunk (decode kernel)
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
    const uint8_t *row = p.kc + blk * p.block_stride + ((key % p.block_size) * p.kv_heads) * width + head_off;
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
      const uint8_t *row = p.vc + blk * p.block_stride + ((kk % p.block_size) * p.kv_heads) * width + head_off;
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

constexpr int kDecChunk = 64;      // key granularity of the decode split (the workspace is sized for it)
constexpr int kDecMaxChunk = 256;
constexpr int kDecWarps = 4;
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecHead = 256;      // head size of the decode kernel
constexpr int kDecBlock = 8;       // keys per MMA step of a warp
// Shared-memory ring of staged K/V words per warp: every lane copies (cp.async,
// 4 bytes at a time: cache rows are only 4-byte aligned) exactly the words it
// later feeds to its MMAs, kDecStages - 1 blocks ahead of the block it computes.
constexpr int kDecStages = 3;
constexpr int kStageK = 17;        // K words per lane: 16 of row g + its scale
constexpr int kStageV = 18;        // V words per lane: 8 of rows 2t and 2t+1 each + their scales
constexpr int kStageWords = (kStageK + kStageV) * 32;  // per warp and stage
constexpr size_t kDecRingBytes = (size_t)kDecWarps * kDecStages * kStageWords * sizeof(uint32_t);

__device__ __forceinline__ void cp_async4(uint32_t *dst, const void *src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void attn_mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void attn_mma1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// Decoded BF16 bits of byte `sel` of `word`, in the high half of the result:
// from this lane's copy of the table (high half = the V value, low half = the
// K value, selected by the caller), or computed with the row's own scale.
template <bool TAB>
__device__ __forceinline__ uint32_t kv_dec(const uint32_t *tab, const float *lut, uint32_t word, int sel, int lane,
                                           float scale, bool value_half) {
  const uint32_t c = (word >> (8 * sel)) & 0xFFu;
  if constexpr (TAB) return value_half ? tab[c * 32 + lane] : tab[c * 32 + lane] << 16;
  else return f32_to_bf16_bits(lut[c] * scale) << 16;
}

// Split-KV decode attention on the tensor cores (mma.sync, BF16 operands,
// FP32 accumulation), for decode batches (one query row per request) of head
// size 256 and GQA groups of 1, 2, 4 or 8.
// CTA = (request b, KV head h, chunk of p.chunk keys); warp w walks keys
// [w * kpw, (w + 1) * kpw) of the chunk 8 at a time:
//   * scores S = Q K^T as one m16n8k16 tile per 16 dims: A = the G query
//     heads (rows >= G zero), B = the decoded K rows.  K-step ks of lane
//     (g, t) takes bytes 16 ks + 4t .. + 3 of key row g (cache rows are only
//     4-byte aligned: 4-byte loads, 16 contiguous bytes per row and
//     instruction), a fixed permutation of the head dimension applied
//     identically to the query fragments;
//   * online softmax per head on the score fragment (lane (g, t) holds head g
//     at keys 2t, 2t+1; the 4 lanes of a head combine by two shuffles),
//     probabilities rounded to BF16;
//   * O^T += V^T P^T as 16 m16n8k8 tiles: A = the decoded V^T tile, B = P^T,
//     which is exactly the score fragment (no data movement).  Lane (g, t)
//     reads 4 bytes (dims 32 r + 4 g .. + 3) of key rows 2t and 2t+1 and
//     packs the two keys per dimension; the 16 output tiles cover the
//     dimensions in a permuted order that the merge undoes;
//   * K and V bytes decode through one lane-replicated table (entry c: BF16 of
//     decode(c) x k_scale in the low half, x v_scale in the high half, for
//     the chunk's first row; conflict-free lookups).  When a row of the chunk
//     carries another scale, the CTA runs the same loop with every byte
//     decoded with its own row's scale, as the reference materialises BF16 K
//     and V;
//   * the next block's K rows are loaded after this block's scores and its V
//     rows after this block's P @ V, so loads overlap the MMAs;
//   * the 4 warps merge in shared memory into one partial (output, max, sum)
//     per head, merged across chunks by attention_combine_kernel, or the
//     output is written directly when one chunk covers the request.
template <int G>
__global__ void __launch_bounds__(kDecThreads) paged_decode_kernel(const AttnArgs p) {
  constexpr int D = kDecHead;
  __shared__ uint32_t kvlut[256 * 32];  // the merge buffer afterwards
  __shared__ float lut[256];
  __shared__ float ks0, vs0;
  __shared__ float wm[kDecWarps][G], wl[kDecWarps][G];
  __shared__ uint32_t wvalid[kDecWarps][kDecStages];  // attended-key mask of each staged block
  extern __shared__ __align__(16) uint32_t dec_ring[];  // [warp][stage][kStageK + kStageV][32 lanes]
  pdl_wait();  // the cache and the queries come from earlier kernels of the stream
  const int b = blockIdx.x / (int)p.kv_heads, h = blockIdx.x - b * (int)p.kv_heads;
  const int split = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = p.q_start[b], q_len = p.q_start[b + 1] - q0;
  const int seq = p.seq_lens[b];
  const int chunk0 = split * p.chunk;
  if (q_len <= 0 || chunk0 >= seq) return;  // the merge reads only chunks that hold keys
  const int64_t width = D + 4;
  const int32_t *table = p.tables + (int64_t)b * p.max_blocks;
  const int bsz = (int)p.block_size;  // < 2^31 (checked by the launcher): 32-bit division
  auto row_of = [&](int key) -> int64_t {  // -1: absent
    if (key >= seq) return -1;
    const int col = key / bsz;
    if (col >= p.max_blocks) return -1;
    const int64_t blk = table[col];
    if (blk < 0 || blk >= p.num_blocks) return -1;
    return blk * p.block_stride + ((int64_t)(key - col * bsz) * p.kv_heads + h) * width;
  };
  for (int i = tid; i < 256; i += kDecThreads) lut[i] = __uint_as_float(g_decode_f32.v[i]);
  // the chunk's reference scales (NaN: no table) and whether every row of
  // the chunk carries them
  float my_k[2], my_v[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int key = chunk0 + tid + kDecThreads * j;
    const int64_t off = key < chunk0 + p.chunk ? row_of(key) : -1;
    my_k[j] = off >= 0 ? __ldg(reinterpret_cast<const float *>(p.kc + off + D)) : 0.f;
    my_v[j] = off >= 0 ? __ldg(reinterpret_cast<const float *>(p.vc + off + D)) : 0.f;
    if (off < 0) my_k[j] = my_v[j] = CUDART_INF_F;  // marks "no row"
  }
  if (tid == 0) {
    ks0 = my_k[0] == CUDART_INF_F ? CUDART_NAN_F : my_k[0];
    vs0 = my_v[0] == CUDART_INF_F ? CUDART_NAN_F : my_v[0];
  }
  __syncthreads();
  const float k_ref = ks0, v_ref = vs0;
  bool same = true;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    same = same && (my_k[j] == CUDART_INF_F || (my_k[j] == k_ref && my_v[j] == v_ref));
  const bool table_ok = __syncthreads_and(same) != 0;
  // warp w fills entries 64 w .. 64 w + 63: lane j computes entry 64 w + 32 i
  // + j, then every entry is broadcast and stored as 32 consecutive words
  auto fill_table = [&]() {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c0 = warp * 64 + i * 32;
      const float dv = lut[c0 + lane];
      const uint32_t mine = f32_to_bf16_bits(dv * k_ref) | (f32_to_bf16_bits(dv * v_ref) << 16);
#pragma unroll 8
      for (int j = 0; j < 32; ++j) kvlut[(c0 + j) * 32 + lane] = __shfl_sync(0xFFFFFFFFu, mine, j);
    }
    __syncthreads();
  };
  if (table_ok) fill_table();

  const int kpw = p.chunk / kDecWarps;  // a multiple of 16
  const int wk0 = chunk0 + warp * kpw;
  const int n_keys = max(0, min(kpw, seq - wk0));
  const int nblk = (n_keys + kDecBlock - 1) / kDecBlock;

  for (int r = 0; r < q_len; ++r) {
    const int64_t tok = q0 + r;
    const int limit = p.causal ? seq - q_len + r : seq - 1;  // last key this row sees
    // query fragments: k-step ks takes dims 16 ks + 4t + {0,1} (a0) and
    // + {2,3} (a2) of head g; rows of heads >= G are zero
    uint32_t qa[16][2];
    {
      const uint16_t *qrow = p.q + (tok * p.heads + (int64_t)h * G + (g < G ? g : 0)) * D;
#pragma unroll
      for (int ks = 0; ks < 16; ++ks) {
        uint2 v = make_uint2(0, 0);
        if (g < G) v = *reinterpret_cast<const uint2 *>(qrow + 16 * ks + 4 * t);
        qa[ks][0] = v.x;
        qa[ks][1] = v.y;
      }
    }
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -CUDART_INF_F, l_run = 0.f;  // of head g

    auto run = [&](auto tab_tag) {
      constexpr bool TAB = decltype(tab_tag)::value;
      uint32_t kr[16];    // K row g: word ks at bytes 16 ks + 4t
      uint32_t vr[8][2];  // V rows 2t, 2t+1: word of dims 32 r + 4g .. + 3
      float ksc = 0.f, vsc[2] = {0.f, 0.f};
      uint32_t *ring = dec_ring + (size_t)warp * kDecStages * kStageWords;
      // cache row of key (lane & 7) of a block (-1: absent) and whether it is
      // attended; the block-table read is issued here, used by stage()
      auto row_pre = [&](int blk, bool &att) -> int64_t {
        const int kk = blk * kDecBlock + (lane & 7);
        const int64_t mine = kk < n_keys ? row_of(wk0 + kk) : -1;
        att = mine >= 0 && wk0 + kk <= limit;
        return mine;
      };
      auto shfl_off = [&](int64_t v, int src) -> int64_t {
        const uint32_t lo = (uint32_t)(uint64_t)v, hi = (uint32_t)((uint64_t)v >> 32);
        return (int64_t)(((uint64_t)__shfl_sync(0xFFFFFFFFu, hi, src) << 32) | __shfl_sync(0xFFFFFFFFu, lo, src));
      };
      // copy this lane's words of block blk into its ring slot; absent keys
      // read row 0 (in bounds) and are masked
      auto stage = [&](int blk, int64_t mine, bool att) {
        const int slot = blk % kDecStages;
        uint32_t *sl = ring + slot * kStageWords;
        const uint32_t valid = __ballot_sync(0xFFFFFFFFu, att) & 0xFFu;
        if (lane == 0) wvalid[warp][slot] = valid;
        const int64_t koff = shfl_off(mine, g);
        const uint8_t *krow = p.kc + (koff >= 0 ? koff : 0);
#pragma unroll
        for (int ks = 0; ks < 16; ++ks) cp_async4(sl + ks * 32 + lane, krow + 16 * ks + 4 * t);
        if (!TAB) cp_async4(sl + 16 * 32 + lane, krow + D);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int64_t voff = shfl_off(mine, 2 * t + j);
          const uint8_t *vrow = p.vc + (voff >= 0 ? voff : 0);
#pragma unroll
          for (int rr = 0; rr < 8; ++rr)
            cp_async4(sl + (kStageK + 2 * rr + j) * 32 + lane, vrow + 32 * rr + 4 * g);
          if (!TAB) cp_async4(sl + (kStageK + 16 + j) * 32 + lane, vrow + D);
        }
      };
      // blocks 0 .. kDecStages - 2 in flight before the first is used; one
      // commit group per block (empty past the last), so waiting for all but
      // the newest kDecStages - 2 groups means the current block has landed
#pragma unroll
      for (int b0 = 0; b0 < kDecStages - 1; ++b0) {
        if (b0 < nblk) {
          bool att;
          const int64_t mine = row_pre(b0, att);
          stage(b0, mine, att);
        }
        cp_async_commit();
      }
      for (int blk = 0; blk < nblk; ++blk) {
        cp_async_wait<kDecStages - 2>();
        __syncwarp();
        const int slot = blk % kDecStages;
        const uint32_t *sl = ring + slot * kStageWords;
        const uint32_t cur_valid = wvalid[warp][slot];
#pragma unroll
        for (int ks = 0; ks < 16; ++ks) kr[ks] = sl[ks * 32 + lane];
        if (!TAB) ksc = __uint_as_float(sl[16 * 32 + lane]);
#pragma unroll
        for (int rr = 0; rr < 8; ++rr)
#pragma unroll
          for (int j = 0; j < 2; ++j) vr[rr][j] = sl[(kStageK + 2 * rr + j) * 32 + lane];
        if (!TAB) {
          vsc[0] = __uint_as_float(sl[(kStageK + 16) * 32 + lane]);
          vsc[1] = __uint_as_float(sl[(kStageK + 17) * 32 + lane]);
        }
        // the block that reuses the slot freed one iteration ago: its table
        // read is in flight during this block's scores
        const int nb = blk + kDecStages - 1;
        bool att_n = false;
        int64_t mine_n = -1;
        if (nb < nblk) mine_n = row_pre(nb, att_n);
        // ---- scores of keys 0..7 of the block (B fragment = K^T: bytes 0,1 ->
        // k-slots 2t, 2t+1; bytes 2,3 -> 2t+8, 2t+9)
        // two accumulators (even and odd k-steps): two dependent MMA chains of
        // 8 instead of one of 16
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 16; ++ks) {
          const uint32_t w = kr[ks];
          const uint32_t b0 = __byte_perm(kv_dec<TAB>(kvlut, lut, w, 0, lane, ksc, false),
                                          kv_dec<TAB>(kvlut, lut, w, 1, lane, ksc, false), 0x7632u);
          const uint32_t b1 = __byte_perm(kv_dec<TAB>(kvlut, lut, w, 2, lane, ksc, false),
                                          kv_dec<TAB>(kvlut, lut, w, 3, lane, ksc, false), 0x7632u);
          attn_mma16816((ks & 1) ? sb : sa, qa[ks][0], qa[ks][1], b0, b1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) sa[q] += sb[q];
        if (nb < nblk) stage(nb, mine_n, att_n);
        cp_async_commit();
        // ---- online softmax of head g over keys 2t, 2t+1
        float s0 = ((cur_valid >> (2 * t)) & 1u) ? sa[0] * p.scale : -CUDART_INF_F;
        float s1 = ((cur_valid >> (2 * t + 1)) & 1u) ? sa[1] * p.scale : -CUDART_INF_F;
        float mb = fmaxf(s0, s1);
        mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, 1));
        mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, 2));
        const float m_new = fmaxf(m_run, mb);
        const float alpha = m_run == -CUDART_INF_F ? 0.f : __expf(m_run - m_new);
        const uint32_t p0 = s0 == -CUDART_INF_F ? 0u : f32_to_bf16_bits(__expf(s0 - m_new));
        const uint32_t p1 = s1 == -CUDART_INF_F ? 0u : f32_to_bf16_bits(__expf(s1 - m_new));
        float ps = bf16_bits_to_f32(p0) + bf16_bits_to_f32(p1);
        ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 1);
        ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 2);
        l_run = l_run * alpha + ps;
        m_run = m_new;
        // ---- O^T = alpha O^T + V^T P^T (columns: heads 2t, 2t+1)
        const float al0 = __shfl_sync(0xFFFFFFFFu, alpha, 8 * t);
        const float al1 = __shfl_sync(0xFFFFFFFFu, alpha, 8 * t + 4);
        if (!__all_sync(0xFFFFFFFFu, al0 == 1.f && al1 == 1.f)) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            o[i][0] *= al0;
            o[i][1] *= al1;
            o[i][2] *= al0;
            o[i][3] *= al1;
          }
        }
        const uint32_t pp = p0 | (p1 << 16);
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            // tile 2 rr + half: row g -> dim 32 rr + 4 g + 2 half, row g + 8 -> + 1
            const uint32_t a0 = __byte_perm(kv_dec<TAB>(kvlut, lut, vr[rr][0], 2 * half, lane, vsc[0], true),
                                            kv_dec<TAB>(kvlut, lut, vr[rr][1], 2 * half, lane, vsc[1], true),
                                            0x7632u);
            const uint32_t a1 = __byte_perm(kv_dec<TAB>(kvlut, lut, vr[rr][0], 2 * half + 1, lane, vsc[0], true),
                                            kv_dec<TAB>(kvlut, lut, vr[rr][1], 2 * half + 1, lane, vsc[1], true),
                                            0x7632u);
            attn_mma1688(o[2 * rr + half], a0, a1, pp);
          }
        }
      }
      cp_async_wait<0>();  // nothing in flight into the ring when the warp moves on
    };
    if (table_ok) run(std::true_type{});
    else run(std::false_type{});

    // ---- merge the warps: lane 4 g (t = 0) owns head g's running max and sum
    __syncthreads();  // every warp is done with the table: its space holds the merge
    if (t == 0 && g < G) {
      wm[warp][g] = m_run;
      wl[warp][g] = l_run;
    }
    float *obuf = reinterpret_cast<float *>(kvlut);  // [kDecWarps][G][D]
#pragma unroll
    for (int rr = 0; rr < 8; ++rr)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int d0 = 32 * rr + 4 * g + 2 * half;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int head = 2 * t + (q & 1), dim = d0 + (q >> 1);
          if (head < G) obuf[(warp * G + head) * D + dim] = o[2 * rr + half][q];
        }
      }
    __syncthreads();
#pragma unroll
    for (int hg = 0; hg < G; ++hg) {
      float M = -CUDART_INF_F;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, wm[w][hg]);
      float ew[kDecWarps], L = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        ew[w] = wm[w][hg] == -CUDART_INF_F ? 0.f : __expf(wm[w][hg] - M);
        L = fmaf(wl[w][hg], ew[w], L);
      }
      const int64_t head = (int64_t)h * G + hg;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int dim = tid + kDecThreads * k;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) acc = fmaf(obuf[(w * G + hg) * D + dim], ew[w], acc);
        if (p.splits == 1) {
          const float inv = L > 0.f ? 1.f / L : 0.f;
          p.out[(tok * p.heads + head) * D + dim] = (uint16_t)f32_to_bf16_bits(acc * inv);
        } else {
          float *dst = p.part + ((tok * p.heads + head) * p.splits + split) * part_stride(D);
          dst[dim] = acc;
          if (tid == 0 && k == 0) {
            dst[D] = M;
            dst[D + 1] = L;
          }
        }
      }
    }
    __syncthreads();  // the buffer is rewritten by the table / the next row
    if (r + 1 < q_len && table_ok) fill_table();
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

// Smallest legal block stride of a cache (one block's bytes), or -1 when the
// block does not fit int64.
static int64_t dense_block_stride(int64_t block_size, int64_t kv_heads, int64_t head_size) {
  int64_t v = 0;
  if (__builtin_mul_overflow(block_size, kv_heads, &v) || __builtin_mul_overflow(v, head_size + 4, &v)) return -1;
  return v;
}

// A block stride the kernels accept: at least one block's bytes, 4-byte
// rows, and every block's last byte addressable in int64.
static bool block_stride_ok(int64_t block_stride, int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                            int64_t head_size) {
  const int64_t dense = dense_block_stride(block_size, kv_heads, head_size);
  int64_t span = 0;
  return dense > 0 && block_stride >= dense && block_stride % 4 == 0 &&
         !__builtin_mul_overflow(num_blocks, block_stride, &span);
}

extern "C" int hif8_kv_cache_write(const void *key, const void *value, int src_dtype, int64_t tokens,
                                   int64_t kv_heads, int64_t head_size, int64_t src_token_stride,
                                   const float *key_scale, const float *value_scale,
                                   const int64_t *slot_mapping, uint8_t *key_cache, uint8_t *value_cache,
                                   int64_t num_blocks, int64_t block_size, int32_t *bad_slots, void *stream) {
  const int64_t dense = dense_block_stride(block_size > 0 ? block_size : 1, kv_heads > 0 ? kv_heads : 1,
                                           head_size > 0 ? head_size : 0);
  return hif8_kv_cache_write_strided(key, value, src_dtype, tokens, kv_heads, head_size, src_token_stride,
                                     key_scale, value_scale, slot_mapping, key_cache, value_cache, num_blocks,
                                     block_size, dense, bad_slots, stream);
}

extern "C" int hif8_kv_cache_write_strided(const void *key, const void *value, int src_dtype, int64_t tokens,
                                           int64_t kv_heads, int64_t head_size, int64_t src_token_stride,
                                           const float *key_scale, const float *value_scale,
                                           const int64_t *slot_mapping, uint8_t *key_cache, uint8_t *value_cache,
                                           int64_t num_blocks, int64_t block_size, int64_t block_stride,
                                           int32_t *bad_slots, void *stream) {
  if (tokens < 0 || kv_heads <= 0 || head_size <= 0 || head_size % 4 != 0 || num_blocks <= 0 ||
      block_size <= 0 || src_token_stride < kv_heads * head_size || src_token_stride % 4 != 0)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (!block_stride_ok(block_stride, num_blocks, block_size, kv_heads, head_size)) return HIF8_ERR_INVALID_ARGUMENT;
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
  p.block_stride = block_stride;
  p.planes = with_v ? 2 : 1;
  p.cache_slots = num_blocks * block_size;
  // 16-element units where the source rows allow 16-byte loads
  const bool vec16 = head_size % 16 == 0 && src_token_stride % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(key) & 15u) == 0 &&
                     (!value || (reinterpret_cast<uintptr_t>(value) & 15u) == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = src_dtype == HIF8_DTYPE_BF16;
  const int64_t group = kv_heads * (head_size + 4);
  const int64_t per_head = head_size / 16;
  if (vec16 && (per_head & (per_head - 1)) == 0 && kv_heads <= kKvScaleSlots && group <= kKvGroupMax) {
    // the warp-per-token kernel: D / 16 a power of two, the row group staged
    KvWarpArgs a{};
    a.p = p;
    a.shift = 0;
    while ((1LL << a.shift) < per_head) ++a.shift;
    a.group = (int)group;
    a.group_stage = (int)((group + 15) / 16 * 16);
    a.store16 = group % 16 == 0 && block_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(key_cache) & 15u) == 0 &&
                (!value_cache || (reinterpret_cast<uintptr_t>(value_cache) & 15u) == 0);
    const size_t smem = 4096 + 2 * kKvScaleSlots * (4 + 4 + 4 + 8) + (size_t)kKvWarps * a.group_stage;
    const int64_t items = p.planes * tokens;
    const int grid = attn_grid_cap((items + kKvWarps - 1) / kKvWarps);
    auto kernel = bf16 ? kv_write_warp_kernel<HIF8_DTYPE_BF16> : kv_write_warp_kernel<HIF8_DTYPE_F16>;
    const int st = ensure_smem_limit(reinterpret_cast<const void *>(kernel), smem);
    if (st != HIF8_OK) return st;
    return launch_pdl(kernel, dim3(grid), dim3(kKvWarps * 32), smem, s, a);
  }
  const int elems = vec16 ? 16 : 4;
  p.units = p.planes * tokens * kv_heads * (head_size / elems);
  if (p.units > 0x7FFFFFFFLL) return HIF8_ERR_INVALID_ARGUMENT;  // 32-bit unit indices
  const int grid = attn_grid_cap((p.units + 255) / 256);  // one wave at most; then kKvUnroll per step
  if (vec16)
    return bf16 ? launch_pdl(kv_write_kernel<HIF8_DTYPE_BF16, 16>, dim3(grid), dim3(256), 0, s, p)
                : launch_pdl(kv_write_kernel<HIF8_DTYPE_F16, 16>, dim3(grid), dim3(256), 0, s, p);
  return bf16 ? launch_pdl(kv_write_kernel<HIF8_DTYPE_BF16, 4>, dim3(grid), dim3(256), 0, s, p)
              : launch_pdl(kv_write_kernel<HIF8_DTYPE_F16, 4>, dim3(grid), dim3(256), 0, s, p);
}

static int attn_nq(int64_t group, int64_t q_rows) { return (int)(group * q_rows); }

// Resident decode CTAs per SM for GQA group g (cached per device).
static int decode_residency(int64_t g) {
  static std::atomic<int> cache[64][4];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  const int gi = g == 1 ? 0 : g == 2 ? 1 : g == 4 ? 2 : 3;
  int v = cache[dev][gi].load(std::memory_order_relaxed);
  if (v == 0) {
    const void *k = gi == 0 ? reinterpret_cast<const void *>(paged_decode_kernel<1>)
                    : gi == 1 ? reinterpret_cast<const void *>(paged_decode_kernel<2>)
                    : gi == 2 ? reinterpret_cast<const void *>(paged_decode_kernel<4>)
                              : reinterpret_cast<const void *>(paged_decode_kernel<8>);
    if (ensure_smem_limit(k, kDecRingBytes) != HIF8_OK ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, kDecThreads, kDecRingBytes) != cudaSuccess || v < 1) {
      cudaGetLastError();
      v = 1;
    }
    cache[dev][gi].store(v, std::memory_order_relaxed);
  }
  return v;
}

// Keys per decode CTA: the multiple of 64 up to 256 that minimises waves of
// resident CTAs x (keys per CTA + a fixed cost of ~32 keys for the table,
// the query load and the merge); ties go to the smaller chunk.
static int decode_chunk(int64_t group, int64_t seq_heads, int64_t max_seq_len) {
  const int64_t slots = (int64_t)num_sms() * decode_residency(group);
  int best = kDecChunk;
  int64_t best_cost = -1;
  for (int c = kDecChunk; c <= kDecMaxChunk; c += 64) {
    const int64_t ctas = seq_heads * ((max_seq_len + c - 1) / c);
    const int64_t cost = ((ctas + slots - 1) / slots) * (c + 32);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

// Sized for the finer of the two kernels' key chunks (the decode kernel's).
// The product is computed with overflow checks: sizes whose partials would
// not fit size_t give SIZE_MAX, which no workspace (and no scratch) meets.
extern "C" size_t hif8_paged_attention_workspace_size(int64_t num_tokens, int64_t num_heads, int64_t head_size,
                                                      int64_t max_seq_len) {
  if (num_tokens <= 0 || num_heads <= 0 || head_size <= 0 || max_seq_len <= 0) return 0;
  const int64_t splits = max_seq_len / kDecChunk + (max_seq_len % kDecChunk != 0);
  if (splits <= 1) return 0;
  size_t bytes = 0;
  if (__builtin_mul_overflow((size_t)num_tokens, (size_t)num_heads, &bytes) ||
      __builtin_mul_overflow(bytes, (size_t)splits, &bytes) ||
      __builtin_mul_overflow(bytes, (size_t)part_stride(head_size), &bytes) ||
      __builtin_mul_overflow(bytes, sizeof(float), &bytes))
    return SIZE_MAX;
  return bytes;
}

namespace hif8 {

int paged_attention_args_status(const void *query, const void *key_cache, const void *value_cache,
                                const void *block_tables, const void *seq_lens, const void *query_start,
                                const void *out, int64_t batch, int64_t num_tokens, int64_t num_heads,
                                int64_t kv_heads, int64_t head_size, int64_t num_blocks, int64_t block_size,
                                int64_t max_blocks, int64_t max_seq_len) {
  if (batch <= 0 || num_tokens < 0 || num_heads <= 0 || kv_heads <= 0 || num_heads % kv_heads != 0 ||
      head_size <= 0 || head_size % 4 != 0 || head_size > 1024 || num_blocks <= 0 || block_size <= 0 ||
      block_size > 0x7FFFFFFFLL || max_blocks <= 0 || max_seq_len < 0)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (!query || !key_cache || !value_cache || !block_tables || !seq_lens || !query_start || !out)
    return HIF8_ERR_INVALID_ARGUMENT;
  if (num_heads / kv_heads > 16) return HIF8_ERR_INVALID_ARGUMENT;
  return HIF8_OK;
}

}  // namespace hif8

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
  const int64_t dense = dense_block_stride(block_size > 0 ? block_size : 1, kv_heads > 0 ? kv_heads : 1,
                                           head_size > 0 ? head_size : 0);
  return hif8_paged_attention_strided(query, key_cache, value_cache, block_tables, seq_lens, query_start, batch,
                                      num_tokens, num_heads, kv_heads, head_size, num_blocks, block_size, dense,
                                      max_blocks, max_seq_len, softmax_scale, causal, out, workspace,
                                      workspace_bytes, stream);
}

extern "C" int hif8_paged_attention_strided(const uint16_t *query, const uint8_t *key_cache,
                                            const uint8_t *value_cache, const int32_t *block_tables,
                                            const int32_t *seq_lens, const int32_t *query_start, int64_t batch,
                                            int64_t num_tokens, int64_t num_heads, int64_t kv_heads,
                                            int64_t head_size, int64_t num_blocks, int64_t block_size,
                                            int64_t block_stride, int64_t max_blocks, int64_t max_seq_len,
                                            float softmax_scale, int causal, uint16_t *out, void *workspace,
                                            size_t workspace_bytes, void *stream) {
  const int args_status =
      paged_attention_args_status(query, key_cache, value_cache, block_tables, seq_lens, query_start, out, batch,
                                  num_tokens, num_heads, kv_heads, head_size, num_blocks, block_size, max_blocks,
                                  max_seq_len);
  if (args_status != HIF8_OK) return args_status;
  if (!block_stride_ok(block_stride, num_blocks, block_size, kv_heads, head_size)) return HIF8_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return HIF8_OK;
  const int64_t group = num_heads / kv_heads;
  const size_t need = hif8_paged_attention_workspace_size(num_tokens, num_heads, head_size, max_seq_len);
  if (need > 0 && (!workspace || workspace_bytes < need)) return HIF8_ERR_WORKSPACE;
  // decode batches (as many query rows as requests) of head size 256 and a
  // power-of-two GQA group take the split-KV decode kernel
  const bool decode = num_tokens == batch && head_size == kDecHead &&
                      (group == 1 || group == 2 || group == 4 || group == 8) &&
                      (reinterpret_cast<uintptr_t>(query) & 7u) == 0 && (reinterpret_cast<uintptr_t>(out) & 3u) == 0;
  const int chunk = decode ? decode_chunk(group, batch * kv_heads, max_seq_len) : kAttnChunk;
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
  p.block_stride = block_stride;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.splits = (int)splits;
  p.chunk = chunk;
  p.scale = softmax_scale;
  p.causal = causal;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // query rows per CTA: every query vector of a CTA shares the key loads
  int status;
  if (decode) {
    const dim3 grid((unsigned)(batch * kv_heads), (unsigned)splits, 1);
    const void *kptr = group == 1   ? reinterpret_cast<const void *>(paged_decode_kernel<1>)
                       : group == 2 ? reinterpret_cast<const void *>(paged_decode_kernel<2>)
                       : group == 4 ? reinterpret_cast<const void *>(paged_decode_kernel<4>)
                                    : reinterpret_cast<const void *>(paged_decode_kernel<8>);
    status = ensure_smem_limit(kptr, kDecRingBytes);
    if (status != HIF8_OK) return status;
    switch (group) {
      case 1: status = launch_pdl(paged_decode_kernel<1>, grid, dim3(kDecThreads), kDecRingBytes, s, p); break;
      case 2: status = launch_pdl(paged_decode_kernel<2>, grid, dim3(kDecThreads), kDecRingBytes, s, p); break;
      case 4: status = launch_pdl(paged_decode_kernel<4>, grid, dim3(kDecThreads), kDecRingBytes, s, p); break;
      default: status = launch_pdl(paged_decode_kernel<8>, grid, dim3(kDecThreads), kDecRingBytes, s, p); break;
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
