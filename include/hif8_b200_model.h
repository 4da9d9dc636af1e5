/*
 * hif8_b200 -- glue kernels of the synthetic Qwen3.5-9B-shaped decoder
 * (configs[4] of the workload) that runs the HiF8 static W8A8KV8 path end to
 * end.  None of these has a counterpart in the reference's operator set: on
 * the reference these steps are vLLM / torch_npu code around the plugin's
 * projections.  They follow transformers' Qwen3_5 text model
 * (models/qwen3_5/modeling_qwen3_5.py): (1 + w) RMSNorm, SiLU-gated MLP,
 * gated attention with q/k RMSNorm and partial rotary embedding, and the
 * gated-delta-net linear attention.
 *
 * Conventions as include/hif8_b200.h: device pointers, a cudaStream_t passed
 * as void*, an int status.  Activations are BF16 (uint16_t bits).
 *
 * Programmatic launch ordering: like the operators of hif8_b200.h, these
 * kernels are launched with programmatic stream serialization, and some
 * let the next programmatic launch of the stream begin before they
 * complete: hif8_model_silu_mul, hif8_model_gate_mul and hif8_model_gdn
 * when their grid is small (decode batches), and
 * hif8_model_peer_allreduce_rmsnorm always.  A kernel of the caller that is
 * itself launched with that attribute right after one of them must wait for
 * the grid dependency (cudaGridDependencySynchronize / griddepcontrol.wait)
 * before it reads their outputs; ordinary launches are unaffected.
 */
#ifndef HIF8_B200_MODEL_H
#define HIF8_B200_MODEL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out = RMSNorm(x [+ residual_in]) * (one_plus ? 1 + w : w), rows x dim,
 * dim % 8 == 0 and dim <= 8192.  With residual_in the BF16 sum is also
 * written to residual_out (the new residual stream). */
int hif8_model_rmsnorm(const uint16_t *x, const uint16_t *residual_in, uint16_t *residual_out,
                       const uint16_t *weight, float eps, int one_plus, int64_t rows, int64_t dim,
                       uint16_t *out, void *stream);

/* out[r, i] = silu(gate_up[r, i]) * gate_up[r, inter + i]. */
int hif8_model_silu_mul(const uint16_t *gate_up, int64_t rows, int64_t inter, uint16_t *out, void *stream);

/* out[i] = x[i] * sigmoid(gate[i]). */
int hif8_model_gate_mul(const uint16_t *x, const uint16_t *gate, int64_t n, uint16_t *out, void *stream);

/* Split a gated-attention projection row [heads x (q | gate) | k | v] into
 * q_out [tokens, heads, head_dim] and k_out / v_out [tokens, kv_heads,
 * head_dim] (q and k: per-head (1 + w) RMSNorm, then rotary embedding of
 * the first rotary_dim dims at positions[token]) and gate_out [tokens,
 * heads * head_dim]. */
int hif8_model_attn_prep(const uint16_t *qkv, int64_t tokens, int heads, int kv_heads, int head_dim,
                         int rotary_dim, const int32_t *positions, const uint16_t *q_norm_w,
                         const uint16_t *k_norm_w, float eps, float rope_theta, uint16_t *q_out,
                         uint16_t *gate_out, uint16_t *k_out, uint16_t *v_out, void *stream);

/* Gated delta net over T tokens of every sequence (T = 1: one decode step).
 * proj rows (batch * T of them, proj_stride elements apart) hold
 * [q: hk*128 | k: hk*128 | v: hv*128 | z: hv*128 | b: hv | a: hv];
 * conv_state [batch, hv, 3, 128, 3] (per value head: the causal-convolution
 * history of its key head's q and k channels and of its own v channels) and
 * rec_state [batch, hv, 128, 128] (FP32) are read and updated in place;
 * out [batch * T, hv * 128]. */
typedef struct Hif8GdnArgs {
  const uint16_t *proj;
  int64_t proj_stride;
  int T;
  int hk, hv;
  int key_dim, value_dim;  /* both 128 */
  const uint16_t *conv_w;  /* [channels, 4] */
  const float *a_log;      /* [hv] */
  const float *dt_bias;    /* [hv] */
  const uint16_t *norm_w;  /* [value_dim] */
  float *conv_state;
  float *rec_state;
  uint16_t *out;
  float eps;
} Hif8GdnArgs;

int hif8_model_gdn(const Hif8GdnArgs *args, int64_t batch, void *stream);

/* ---- glue fused into the decode-step projection --------------------------
 * One launch of the fused static quant + GEMV (rows m <= 8, k % 256 == 0,
 * weight 32-byte aligned, BF16 tensors 16-byte aligned, BF16 out [m, n])
 * whose quantised activation is produced in its prologue:
 *   HIF8_GLUE_SILU_MUL: silu(x[:, :k]) * x[:, k:2k]              (x [m, 2k])
 *   HIF8_GLUE_GATE_MUL: x * sigmoid(aux)                         (x, aux [m, k])
 *   HIF8_GLUE_RMSNORM:  RMSNorm(x + aux) * (one_plus ? 1 + w : w) (aux may be
 *                       NULL; with aux, residual_out (may be NULL) receives
 *                       the BF16 sum x + aux)
 * each rounded to BF16 exactly as the separate glue kernels above round it
 * (the RMSNorm's sum of squares is reduced in another order), then encoded
 * with fixed_scale[0] as hif8_static_quant does and multiplied with the HiF8
 * weight as soft_hif8_static_fused_gemm does.  Shapes the persistent kernel
 * cannot plan return HIF8_ERR_INVALID_ARGUMENT. */
#define HIF8_GLUE_SILU_MUL 1
#define HIF8_GLUE_GATE_MUL 2
#define HIF8_GLUE_RMSNORM 3

typedef struct Hif8GlueArgs {
  int kind;
  const uint16_t *aux;     /* gate (GATE_MUL) / residual (RMSNORM) */
  uint16_t *residual_out;  /* RMSNORM: x + aux */
  const uint16_t *norm_w;  /* RMSNORM: [k] */
  float eps;
  int one_plus;
} Hif8GlueArgs;

int hif8_model_glue_linear(const uint16_t *x, const Hif8GlueArgs *glue, int64_t m, int64_t k,
                           const uint8_t *weight, const float *fixed_scale, const float *channel_scale,
                           int64_t n, uint16_t *out, void *stream);

/* ---- tensor-parallel all-reduce (fused with residual + RMSNorm) ---------
 * Replaces NCCL all-reduce (+ RMSNorm) after every row-parallel projection
 * of a decode step.  Every rank owns one device buffer (hif8_peer_alloc) of
 * hif8_peer_buffer_bytes(world, max_rows, dim) bytes that its peers map over
 * NVLink (hif8_peer_open of the exchanged 64-byte IPC handle).  Layout of a
 * rank's buffer: two slots, each holding `world` partials of max_rows x dim
 * FP32 (partial q = rank q's), then one uint32 flag per (source rank, CTA)
 * for up to 16 CTAs, then the rank's own scratch (row sums of squares and
 * two counters, never written by peers).  One launch per rank, of C CTAs
 * (one per 128 KB that the rank pushes, rows x dim x 4 x world bytes, at
 * most 16 and at most dim / 128); CTA c owns the column slice [c dim / C,
 * (c + 1) dim / C) of every row:
 *   1. stores the slice of this rank's partial `local` (rows x dim; FP32,
 *      the unrounded output of hif8_linear_partial_f32 /
 *      hif8_static_fused_linear_partial_f32, or BF16, widened) as FP32 into
 *      partial [rank] of the slot in every rank's buffer (its own first):
 *      one-way peer stores, from C SMs;
 *   2. system-scope fence, then writes epoch into flag[rank][c] of every
 *      rank's buffer, and waits (bounded by timeout_ns of %globaltimer; on
 *      time-out *error = 1 and the kernel finishes) until flag[q][c] of its
 *      own buffer has reached epoch for every rank q;
 *   3. sums the ranks' partials of the slice in FP32 from its own buffer in
 *      rank order (identical on every rank) and rounds the sum to BF16
 *      once; with `weight` it adds the residual (BF16) and normalises: out =
 *      RMSNorm(sum + residual) * (one_plus ? 1 + w : w), residual_out = sum
 *      + residual, the row norm from the CTAs' row sums of squares added in
 *      CTA order after a bounded barrier of the grid (identical on every
 *      CTA and rank); with weight == NULL, out = the sum.
 * dim % 256 == 0; with weight, rows <= 8.
 * epoch = *epoch_counter + 1 (a per-rank device counter, advanced by the
 * launch's last CTA), so the launch can live in a CUDA graph.  Two slots
 * (alternate call sites) keep a rank from overwriting partials a slower
 * peer still reads.  Plain peer loads and stores only (no multicast).  The
 * CTAs signal programmatic dependents at their start (see hif8_b200.h on
 * the ordering contract). */
size_t hif8_peer_buffer_bytes(int64_t world, int64_t max_rows, int64_t dim);

typedef struct Hif8PeerArgs {
  const void *local;              /* this rank's partial, rows x dim, in local_dtype */
  const uint16_t *residual;       /* may be NULL */
  const uint16_t *weight;         /* [dim] */
  uint16_t *out, *residual_out;   /* rows x dim each */
  uint8_t *const *peer_buf;       /* device array [world] of buffer bases (own + mapped peers) */
  uint32_t *epoch_counter;        /* this rank's device counter */
  int *error;                     /* this rank's device error word */
  int64_t rows, dim, max_rows;
  int rank, world, slot, one_plus;
  float eps;
  uint64_t timeout_ns;
  int local_dtype;                /* HIF8_DTYPE_F32 (an unrounded partial) or HIF8_DTYPE_BF16 */
} Hif8PeerArgs;

int hif8_model_peer_allreduce_rmsnorm(const Hif8PeerArgs *args, void *stream);

/* Peer buffers: cudaMalloc'd device memory with its IPC handle (64 bytes),
 * a mapping of a peer's handle, and the release of either. */
int hif8_peer_alloc(size_t bytes, void **ptr, void *handle64);
int hif8_peer_open(const void *handle64, void **ptr);
int hif8_peer_close(void *ptr, int opened);

#ifdef __cplusplus
}
#endif

#endif /* HIF8_B200_MODEL_H */
