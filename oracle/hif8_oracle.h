/*
 * CPU oracle for the HiFloat8 (HiF8) static W8A8KV8 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * kernels are compared against; it is never linked into, loaded by or called
 * from the product path (the hif8_b200 package).  Only tests/, the smoke()
 * entry of __graft_entry__.py and bench.py's cpu_baseline / --impl reference
 * legs may load it.
 *
 * It restates, in plain C, the reference plugin's CPU codec and its static
 * quantisation / KV-page contracts (reference paths are relative to the
 * reference project root):
 *   - src/vllm_ascend_hif8/codec.py            byte layout, encode_ascend, decode table
 *   - src/vllm_ascend_hif8/torch_codec.py      4096-entry exponent/top-mantissa encode LUT
 *   - src/vllm_ascend_hif8/calibration.py      saturating_encode_tensor / static_quantize_tensor
 *   - src/vllm_ascend_hif8/kv_cache.py         pack_kv_rows / scatter_kv_rows / gather_kv_rows
 *   - src/vllm_ascend_hif8/reference.py        linear_u8_u8 (FP64 accumulation)
 *
 * Parity of this restatement is pinned against golden vectors produced by the
 * reference's own Python code (tests/golden/make_golden.py).
 */
#ifndef HIF8_ORACLE_H
#define HIF8_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scalar encode of one FP32 value, nearest / ties away from zero
 * (codec.py:148-180). */
uint8_t hif8o_encode_value(float value);

/* Decode one byte to its exact value (codec.py:90-103). */
float hif8o_decode_value(uint8_t byte);

/* BF16 payload of a decoded byte; NaN is 0x7FC0 (codec.py:106-145). */
uint16_t hif8o_decode_bf16_bits(uint8_t byte);

/* Fill the 256-entry decode table (FP32). */
void hif8o_decode_table(float out[256]);

/* The 4096-entry magnitude LUT indexed by (fp32 exponent << 4) | top-4
 * mantissa bits (torch_codec.py:19-29). */
void hif8o_encode_lut4096(uint8_t out[4096]);

/* Tensor encode with the LUT semantics of torch_codec.encode_tensor
 * (torch_codec.py:32-49). */
void hif8o_encode_tensor(const float *x, int64_t n, uint8_t *out);

/* Static quantisation (calibration.py:139-201):
 *   q = fp32(x[r, k]) / scale[r % scale_count]   (IEEE division)
 *   q = clamp(q, -32768, 32768) if q is finite
 *   out[r, k] = encode_tensor(q)
 * x_dtype: 0 = FP16 bits, 1 = BF16 bits.  row_scale (may be NULL) receives
 * scale[r % scale_count] for every row. */
/* Dynamic per-row quant (codec.py:205-255): scale = max(finite amax,
 * 1e-12), codes of x / scale with a double-precision quotient. */
void hif8o_dynamic_quant(const uint16_t *x, int x_dtype, int64_t rows, int64_t k, uint8_t *out,
                         float *row_scale);

void hif8o_static_quant(const uint16_t *x, int x_dtype, int64_t rows, int64_t k,
                        const float *scale, int64_t scale_count, uint8_t *out,
                        float *row_scale);

/* Scaled decode: out[r, k] = bf16_rne(decode(data[r, k]) * scale[r]),
 * NaN -> 0x7FC0 (the behaviour pinned by tests/test_npu_ops.py:90-135 of the
 * reference).  row_stride is in bytes. */
void hif8o_scaled_decode(const uint8_t *data, int64_t rows, int64_t k, int64_t row_stride,
                         const float *scale, uint16_t *out);

/* Round FP32 to BF16 bits, nearest-even; NaN -> 0x7FC0 (torch's c10 rule). */
uint16_t hif8o_f32_to_bf16_bits(float v);

/* Round FP32 to FP16 bits, nearest-even (IEEE). */
uint16_t hif8o_f32_to_f16_bits(float v);

/* FP16 / BF16 bits to FP32. */
float hif8o_f16_bits_to_f32(uint16_t h);
float hif8o_bf16_bits_to_f32(uint16_t h);

/* Fused static KV write, the contract of kv_runtime._write_hif8_cache
 * (kv_runtime.py:1222-1339) = static quant per head (S = heads) + pack_kv_rows
 * (kv_cache.py:151-170) + slot-mapping scatter (kv_cache.py:187-218).
 * src: [tokens, heads, head_size] FP16/BF16 bits; cache: [blocks, block_size,
 * heads, head_size + 4] bytes.  Negative slots are skipped; slots whose block
 * is outside the cache are skipped and counted in the return value. */
int64_t hif8o_kv_write(const uint16_t *src, int src_dtype, int64_t tokens, int64_t heads,
                       int64_t head_size, const float *head_scale, const int64_t *slot_mapping,
                       uint8_t *cache, int64_t num_blocks, int64_t block_size);

/* Decoded U8 x U8 linear with FP64 accumulation and the epilogue
 * acc * a_scale * w_scale + bias (reference.py:10-43).  bias may be NULL. */
void hif8o_linear_f64(const uint8_t *a, const uint8_t *w, const float *a_scale,
                      const float *w_scale, const float *bias, int64_t m, int64_t n,
                      int64_t k, double *out);

#ifdef __cplusplus
}
#endif

#endif /* HIF8_ORACLE_H */
