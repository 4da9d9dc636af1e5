/*
 * hif8_b200 -- C ABI of the B200 (sm_100a) HiFloat8 static W8A8KV8 hot path.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*, i.e. a
 * cudaStream_t; NULL = legacy default stream).  Every entry point enqueues
 * its kernels asynchronously on that stream and returns a status code
 * (HIF8_OK on success).  No entry point allocates device memory: outputs and
 * (where a workspace is named) the scratch buffer are owned by the caller.
 * Device pointers must be on the current CUDA device.
 *
 * Each entry point replaces one operator of the reference plugin; the cited
 * lines are in the reference project (csrc/extension/ is its ACLNN bridge,
 * src/vllm_ascend_hif8/ its Python layer).
 *
 * Kernels are launched with programmatic stream serialization (set
 * HIF8_DISABLE_PDL=1 to turn it off), and hif8_static_quant may let the next
 * programmatic launch of the stream begin before it completes.  A kernel of
 * the caller that is itself launched with that attribute right after one of
 * these entry points must wait for the grid dependency
 * (cudaGridDependencySynchronize / griddepcontrol.wait) before it reads
 * their outputs; ordinary launches are unaffected.
 */
#ifndef HIF8_B200_H
#define HIF8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
#define HIF8_OK 0
#define HIF8_ERR_INVALID_ARGUMENT 1 /* shape/dtype/pointer contract violated */
#define HIF8_ERR_CUDA 2             /* a CUDA runtime call or launch failed */
#define HIF8_ERR_WORKSPACE 3        /* workspace missing or too small */

/* ---- dtype codes (match the reference bridge: kFp16Output = 0,
 *      kBf16Output = 1, csrc/extension/hif8_native.cpp:32-33) ---------- */
#define HIF8_DTYPE_F16 0
#define HIF8_DTYPE_BF16 1
#define HIF8_DTYPE_NONE -1 /* "no bias" */
#define HIF8_DTYPE_F32 2   /* FP32: output of the tensor-parallel partial products only */

/* Human-readable text for a status code. */
const char *hif8_status_string(int status);

/* Text of the last CUDA error seen by this library on the calling thread
 * (valid after HIF8_ERR_CUDA). */
const char *hif8_last_error(void);

/* Library version, e.g. "0.1.0". */
const char *hif8_version(void);

/* ---- codec tables (host-side, no device work) ---------------------- */

/* 256 BF16 payloads of the HiF8 decode; NaN byte -> 0x7FC0.
 * Replaces the generated decode tables of src/vllm_ascend_hif8/tablegen.py:63-82. */
void hif8_decode_table_bf16(uint16_t out[256]);

/* 4096-entry magnitude encode LUT indexed by (fp32 exponent << 4) | top-4
 * mantissa bits.  Same contents as torch_codec.FLOAT32_ENCODE_LUT
 * (src/vllm_ascend_hif8/torch_codec.py:19-29). */
void hif8_encode_table(uint8_t out[4096]);

/* ---- activation static quantisation --------------------------------
 * Replaces op hif8_static_quant (csrc/extension/pybind.cpp:8,
 * csrc/extension/hif8_native.cpp:487-554, kernel
 * csrc/opp/op_kernel/hif8_static_quant.cpp).
 *   data[r, k]   = enc_sat( fp32(x[r, k]) / fixed_scale[r % scale_count] )
 *   row_scale[r] = fixed_scale[r % scale_count]        (row_scale may be NULL)
 * x: [rows, k] contiguous FP16/BF16 (x_dtype); data: [rows, k] bytes.
 * IEEE division, finite values saturate to +-32768, NaN -> 0x80, +-Inf ->
 * 0x6F/0xEF: bit-exact with calibration.static_quantize_tensor. */
int hif8_static_quant(const void *x, int x_dtype, int64_t rows, int64_t k,
                      const float *fixed_scale, int64_t scale_count, uint8_t *data,
                      float *row_scale, void *stream);

/* ---- scaled decode ----------------------------------------------------
 * Replaces op hif8_scaled_decode (csrc/extension/pybind.cpp:9,
 * csrc/extension/hif8_native.cpp:556-611).
 *   out[r, k] = bf16_rne( decode(data[r * data_row_stride + k]) * scale[r] ),
 * NaN -> 0x7FC0.  out: [rows, k] contiguous BF16 bits.  data_row_stride is in
 * bytes (>= k), so KV page rows with their 4-byte sidecar decode in place. */
int hif8_scaled_decode(const uint8_t *data, int64_t rows, int64_t k, int64_t data_row_stride,
                       const float *scale, uint16_t *out, void *stream);

/* ---- embedding gather-decode --------------------------------------------
 * Replaces the HiF8 token-embedding lookup of the W8A8HIF8_SOFT scheme
 * (src/vllm_ascend_hif8/scheme.py:120-131: index_select of the requested
 * rows and scales, BF16 decode table, BF16 product).
 *   out[t, j] = bf16_rne( decode(weight[ids[t], j]) * bf16_rne(weight_scale[ids[t]]) ),
 * NaN -> 0x7FC0.  weight: [vocab, k] bytes (row-major), weight_scale: [vocab]
 * FP32, ids: [n] int64, out: [n, k] contiguous BF16 bits.  Only the requested
 * rows are read.  Ids outside [0, vocab) give zero rows and are counted into
 * *bad_ids (device int32, may be NULL). */
int hif8_embedding_gather(const uint8_t *weight, const float *weight_scale, int64_t vocab, int64_t k,
                          const int64_t *ids, int64_t n, uint16_t *out, int32_t *bad_ids, void *stream);

/* ---- linear -------------------------------------------------------------
 * y[m, n] = cast( (acc[m, n] * channel_scale[n]) * token_scale[m] + bias[n] ),
 * acc = sum_k decode(activation[m, k]) * decode(weight[n, k]) in FP32.
 * activation: [m, k] bytes, weight: [n, k] bytes (row-major, K contiguous),
 * bias: [n] FP16/BF16 or NULL (bias_dtype HIF8_DTYPE_NONE), out: [m, n] in
 * output_dtype.
 *
 * soft_hif8_gemv replaces op soft_hif8_gemv (csrc/extension/pybind.cpp:10,
 * hif8_native.cpp:613-631) and keeps its contract m <= 2.
 * soft_hif8_gemm replaces ops soft_hif8_gemm / soft_hif8_prefill_gemm
 * (csrc/extension/pybind.cpp:11, hif8_native.cpp:633-669), any m >= 1; small
 * m runs the split-K tensor-core GEMV, large m the tcgen05 GEMM.
 * workspace: soft_hif8_gemm_workspace_size() bytes of device memory, 256-byte
 * aligned (may be NULL when that size is 0); it holds the BF16 copy of the
 * activation that the tensor-memory accelerator streams, and one error word. */
int soft_hif8_gemv(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                   const float *channel_scale, const void *bias, int bias_dtype,
                   int output_dtype, int64_t m, int64_t n, int64_t k, void *out, void *stream);

size_t soft_hif8_gemm_workspace_size(int64_t m, int64_t n, int64_t k);

int soft_hif8_gemm(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                   const float *channel_scale, const void *bias, int bias_dtype,
                   int output_dtype, int64_t m, int64_t n, int64_t k, void *out,
                   void *workspace, size_t workspace_bytes, void *stream);

/* ---- dynamic path (W8A8HIF8_SOFT checkpoints) ----------------------------
 * hif8_dynamic_quant replaces op hif8_dynamic_quant (csrc/extension/
 * pybind.cpp:58, hif8_native.cpp:433-486, kernel csrc/opp/op_kernel/
 * hif8_dynamic_quant.cpp:11-221; CPU rule codec.py:205-255): per row r,
 * scale = max(amax of the row's finite |x|, 1e-12) and data = the HiF8 code
 * of x / scale (nearest, ties away; NaN and Inf keep their codes), bit-exact
 * with the reference's double-precision quotient.  x: [rows, k] FP16/BF16
 * (x_dtype); data: [rows, k]; row_scale[r * scale_stride] receives the scale
 * (the reference returns it as a stride-16 view).
 * soft_hif8_fused_gemm replaces op soft_hif8_fused_gemm (pybind.cpp:12,
 * hif8_native.cpp:676-760): the dynamic quant of x followed by the linear
 * (bit-identical to hif8_dynamic_quant + soft_hif8_gemm), m <= 2 as the
 * reference; workspace: soft_hif8_fused_gemm_workspace_size() bytes, 256-byte
 * aligned (the codes and row scales). */
int hif8_dynamic_quant(const void *x, int x_dtype, int64_t rows, int64_t k, uint8_t *data,
                       float *row_scale, int64_t scale_stride, void *stream);

size_t soft_hif8_fused_gemm_workspace_size(int64_t m, int64_t n, int64_t k);

int soft_hif8_fused_gemm(const void *x, int x_dtype, const uint8_t *weight, const float *channel_scale,
                         const void *bias, int bias_dtype, int output_dtype, int64_t m, int64_t n,
                         int64_t k, void *out, void *workspace, size_t workspace_bytes, void *stream);

/* ---- the static scheme's apply in one call ---------------------------
 * hif8_static_linear replaces the pair of operator calls that the static
 * scheme's apply makes per projection (reference src/vllm_ascend_hif8/
 * scheme.py:174-211): for m <= fused_max_rows (at most 4) the fused quant +
 * linear of soft_hif8_static_fused_gemm, otherwise hif8_static_quant of x
 * with the one input_scale into the workspace followed by soft_hif8_gemm --
 * the same kernels and bytes as the two separate calls.  x: [m, k]
 * FP16/BF16 (x_dtype); input_scale: one float (device); bias optional;
 * out: [m, n] of output_dtype.  workspace: hif8_static_linear_workspace_size()
 * bytes, 256-byte aligned (0 bytes, and NULL allowed, on the fused path). */
size_t hif8_static_linear_workspace_size(int64_t m, int64_t n, int64_t k, int fused_max_rows);

int hif8_static_linear(const void *x, int x_dtype, const uint8_t *weight, const float *input_scale,
                       const float *channel_scale, const void *bias, int bias_dtype, int output_dtype, int64_t m,
                       int64_t n, int64_t k, int fused_max_rows, void *out, void *workspace, size_t workspace_bytes,
                       void *stream);

/* ---- tensor-parallel partial products ---------------------------------
 * No counterpart in the reference, which runs a projection on one device.
 * When a row-parallel projection is split over ranks by its input columns,
 * every rank's partial product must be summed before it is rounded: these
 * write the partial y[m, n] = (acc[m, n] * channel_scale[n]) * ts[m] as
 * FP32 (no bias, no rounding), so the ranks' partials summed in FP32 and
 * rounded to BF16 once give the unsharded projection's output up to the
 * order of the FP32 sums (rounding each partial to BF16 first moves
 * elements by an ulp, and a static HiF8 quantisation downstream turns such
 * an ulp into a whole code step).
 * hif8_linear_partial_f32: HiF8 activation bytes + token scales, any m;
 * workspace as soft_hif8_gemm (soft_hif8_gemm_workspace_size; out 16-byte
 * aligned for the tcgen05 path).
 * hif8_static_fused_linear_partial_f32: FP16/BF16 x (x_dtype) statically
 * quantised with fixed_scale[0] inside the kernel, m <= 8. */
int hif8_linear_partial_f32(const uint8_t *activation, const uint8_t *weight, const float *token_scale,
                            const float *channel_scale, int64_t m, int64_t n, int64_t k, float *out,
                            void *workspace, size_t workspace_bytes, void *stream);

int hif8_static_fused_linear_partial_f32(const void *x, int x_dtype, const uint8_t *weight,
                                         const float *fixed_scale, const float *channel_scale, int64_t m,
                                         int64_t n, int64_t k, float *out, void *stream);

/* ---- fused static quant + linear ---------------------------------------
 * Replaces op soft_hif8_static_fused_gemm (csrc/extension/pybind.cpp:13,
 * hif8_native.cpp:784-...): x FP16/BF16 [m, k] is encoded with the single
 * fixed_scale[0] (bytes identical to hif8_static_quant), decoded, and fed to
 * the linear above with token_scale = fixed_scale[0].  Contract m <= 4. */
int soft_hif8_static_fused_gemm(const void *x, int x_dtype, const uint8_t *weight,
                                const float *fixed_scale, const float *channel_scale,
                                const void *bias, int bias_dtype, int output_dtype,
                                int64_t m, int64_t n, int64_t k, void *out, void *stream);

/* ---- paged HiF8 KV cache -----------------------------------------------
 * Page layout (src/vllm_ascend_hif8/kv_cache.py:26-88): K and V caches are
 * separate byte tensors [num_blocks, block_size, kv_heads, head_size + 4];
 * each row is head_size HiF8 bytes followed by its little-endian FP32 scale.
 *
 * hif8_kv_cache_write replaces the static write path
 * kv_runtime._write_hif8_cache (src/vllm_ascend_hif8/kv_runtime.py:1222-1339):
 * static quant with per-head scales (S = kv_heads), pack_kv_rows
 * (kv_cache.py:151-170) and the slot_mapping index_copy_, fused in one
 * kernel.  key/value: [tokens, kv_heads, head_size] FP16/BF16 (src_dtype),
 * row stride src_token_stride elements between tokens (>= kv_heads*head_size);
 * slot_mapping: [tokens] int64, negative = skip.  Rows whose block is outside
 * [0, num_blocks) are skipped and counted into *bad_slots (device int32, may
 * be NULL). value/value_cache/value_scale may be NULL to write K only. */
int hif8_kv_cache_write(const void *key, const void *value, int src_dtype, int64_t tokens,
                        int64_t kv_heads, int64_t head_size, int64_t src_token_stride,
                        const float *key_scale, const float *value_scale,
                        const int64_t *slot_mapping, uint8_t *key_cache, uint8_t *value_cache,
                        int64_t num_blocks, int64_t block_size, int32_t *bad_slots,
                        void *stream);

/* hif8_kv_cache_write for caches whose consecutive blocks are block_stride
 * bytes apart (hif8_kv_cache_write is this with the dense stride
 * block_size * kv_heads * (head_size + 4)).  block_stride >= that, a
 * multiple of 4, and num_blocks * block_stride must fit int64_t.  vLLM's
 * block-major page [num_blocks][2][block_size][kv_heads][head_size + 4]
 * (K rows, then V rows) is key_cache = page base, value_cache = base + one
 * block image, block_stride = its page size.  Replaces the same reference
 * write path as hif8_kv_cache_write, for the cache tensors vLLM binds
 * (kv_runtime.py:533-571 _bind_hif8_cache_tensors). */
int hif8_kv_cache_write_strided(const void *key, const void *value, int src_dtype, int64_t tokens,
                                int64_t kv_heads, int64_t head_size, int64_t src_token_stride,
                                const float *key_scale, const float *value_scale,
                                const int64_t *slot_mapping, uint8_t *key_cache, uint8_t *value_cache,
                                int64_t num_blocks, int64_t block_size, int64_t block_stride,
                                int32_t *bad_slots, void *stream);

/* Paged attention over HiF8 pages; replaces _gather_dense_hif8 + scaled
 * decode + the fused-infer-attention call of kv_runtime.py:1375-1563 (and the
 * oracle kv_cache.paged_attention_reference, kv_cache.py:314-372).  Only the
 * pages a request touches are read; K/V are decoded in registers (value
 * rounded to BF16, as the reference materialises them), softmax in FP32.
 *   query: [num_tokens, num_heads, head_size] BF16, tokens of request b are
 *          rows [query_start[b], query_start[b+1]) and sit at the last
 *          positions of that request's context (right-aligned causal mask);
 *   block_tables: [batch, max_blocks] int32; seq_lens: [batch] int32, each
 *          <= max_seq_len; table entries outside [0, num_blocks) are skipped;
 *   query_start: [batch + 1] int32 (cumulative); out: like query.
 * workspace: hif8_paged_attention_workspace_size() bytes (split-KV partials;
 * the size function returns SIZE_MAX where that product overflows size_t, so
 * such a call gets HIF8_ERR_WORKSPACE). */
size_t hif8_paged_attention_workspace_size(int64_t num_tokens, int64_t num_heads,
                                           int64_t head_size, int64_t max_seq_len);

int hif8_paged_attention(const uint16_t *query, const uint8_t *key_cache,
                         const uint8_t *value_cache, const int32_t *block_tables,
                         const int32_t *seq_lens, const int32_t *query_start, int64_t batch,
                         int64_t num_tokens, int64_t num_heads, int64_t kv_heads,
                         int64_t head_size, int64_t num_blocks, int64_t block_size,
                         int64_t max_blocks, int64_t max_seq_len, float softmax_scale, int causal,
                         uint16_t *out, void *workspace, size_t workspace_bytes, void *stream);

/* hif8_paged_attention over caches whose consecutive blocks are
 * block_stride bytes apart (same rule as hif8_kv_cache_write_strided; K and
 * V share the stride).  hif8_paged_attention is this with the dense stride. */
int hif8_paged_attention_strided(const uint16_t *query, const uint8_t *key_cache,
                                 const uint8_t *value_cache, const int32_t *block_tables,
                                 const int32_t *seq_lens, const int32_t *query_start, int64_t batch,
                                 int64_t num_tokens, int64_t num_heads, int64_t kv_heads,
                                 int64_t head_size, int64_t num_blocks, int64_t block_size,
                                 int64_t block_stride, int64_t max_blocks, int64_t max_seq_len,
                                 float softmax_scale, int causal, uint16_t *out, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* hif8_paged_attention without a caller workspace.  No counterpart in the
 * reference (its attention scratch comes from the framework allocator).
 * For callers that cannot hand out device memory per call: a C host that
 * only receives tensors and a stream from its framework, or an engine that
 * has reserved all free HBM for its KV-page pool.  The split-KV partials go
 * to a fixed per-device scratch array inside this library:
 *  - at most HIF8_NOALLOC_ATTENTION_SCRATCH_BYTES (8 MiB) per call, as
 *    hif8_paged_attention_workspace_size() counts it; larger calls return
 *    HIF8_ERR_WORKSPACE and enqueue nothing;
 *  - the scratch need not start at zero (each call writes every partial it
 *    reads);
 *  - calls in flight at the same time on one device (other streams, or host
 *    threads without ordering) race on the shared scratch; calls on one
 *    stream are ordered and safe;
 *  - the first call on each device looks the scratch address up with
 *    cudaGetSymbolAddress, with that device current; make it before any
 *    stream capture.
 * Arguments are checked first, as hif8_paged_attention checks them (a bad
 * call gets HIF8_ERR_INVALID_ARGUMENT at any size); other arguments and
 * errors as hif8_paged_attention. */
#define HIF8_NOALLOC_ATTENTION_SCRATCH_BYTES ((size_t)8 << 20)
int hif8_paged_attention_noalloc(const uint16_t *query, const uint8_t *key_cache,
                                 const uint8_t *value_cache, const int32_t *block_tables,
                                 const int32_t *seq_lens, const int32_t *query_start, int64_t batch,
                                 int64_t num_tokens, int64_t num_heads, int64_t kv_heads,
                                 int64_t head_size, int64_t num_blocks, int64_t block_size,
                                 int64_t max_blocks, int64_t max_seq_len, float softmax_scale,
                                 int causal, uint16_t *out, void *stream);

/* Gather + decode the rows of every request into a dense BF16 tensor, the
 * output of kv_runtime._gather_dense_hif8 (kv_runtime.py:1375-1468):
 * out[sum_b seq_lens[b], kv_heads, head_size] with out_start[b] the first
 * row of request b (cumulative, [batch + 1]).  Positions whose block-table
 * entry is outside [0, num_blocks) decode to zeros. */
int hif8_kv_gather_decode(const uint8_t *cache, const int32_t *block_tables,
                          const int32_t *seq_lens, const int32_t *out_start, int64_t batch,
                          int64_t kv_heads, int64_t head_size, int64_t num_blocks,
                          int64_t block_size, int64_t max_blocks, int64_t max_seq_len,
                          uint16_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* HIF8_B200_H */
