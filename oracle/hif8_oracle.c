/*
 * CPU oracle for the HiFloat8 static W8A8KV8 hot path -- TEST INFRASTRUCTURE.
 *
 * Never part of the product: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline legs load this library, as the checker.
 *
 * Every function restates a function of the reference plugin (paths relative
 * to the reference project root; line numbers cited per function).  Compile
 * without -ffast-math and with -ffp-contract=off: the static quantiser relies
 * on correctly rounded IEEE single-precision division, exactly like
 * `x.to(torch.float32) / divisor` in calibration.py:201.
 */
#include "hif8_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define HIF8_NAN 0x80u
#define HIF8_PINF 0x6Fu
#define HIF8_NINF 0xEFu
#define HIF8_MAX_FINITE 32768.0
#define HIF8_UNDERFLOW_TIE (1.0 / 8388608.0) /* 2^-23 */
#define HIF8_OVERFLOW_TIE 40960.0            /* 1.25 * 2^15 */

typedef struct {
    double value;
    uint8_t code;
} hif8o_entry;

static hif8o_entry g_positive[127];
static int g_positive_ready = 0;
static float g_decode[256];
static uint8_t g_lut4096[4096];
static int g_tables_ready = 0;

/* codec.py:27-49 -- lower seven bits of a finite normal value. */
static int normal_code(int exponent, int mantissa_index) {
    if (exponent >= -3 && exponent <= 3) {
        static const int base_by_exponent[7] = {0x38, 0x30, 0x18, 0x08, 0x10, 0x20, 0x28};
        return base_by_exponent[exponent + 3] + mantissa_index;
    }
    if (exponent >= 4 && exponent <= 7) return 0x40 + (exponent - 4) * 0x04 + mantissa_index;
    if (exponent >= -7 && exponent <= -4) return 0x50 + (-exponent - 4) * 0x04 + mantissa_index;
    if (exponent >= 8 && exponent <= 15) return 0x60 + (exponent - 8) * 0x02 + mantissa_index;
    return 0x70 + (-exponent - 8) * 0x02 + mantissa_index; /* -15 .. -8 */
}

/* codec.py:52-60 */
static int mantissa_bits(int exponent) {
    int a = exponent < 0 ? -exponent : exponent;
    if (a <= 3) return 3;
    if (a <= 7) return 2;
    return 1;
}

static int cmp_entry(const void *a, const void *b) {
    double x = ((const hif8o_entry *)a)->value, y = ((const hif8o_entry *)b)->value;
    return (x > y) - (x < y);
}

/* codec.py:63-82 -- the 127 non-negative finite values, sorted. */
static void build_positive(void) {
    if (g_positive_ready) return;
    int n = 0;
    g_positive[n].value = 0.0;
    g_positive[n++].code = 0x00;
    for (int e = -22; e < -15; ++e) {
        g_positive[n].value = ldexp(1.0, e);
        g_positive[n++].code = (uint8_t)(e + 23);
    }
    for (int e = -15; e < 16; ++e) {
        int mb = mantissa_bits(e);
        for (int i = 0; i < (1 << mb); ++i) {
            double v = (1.0 + (double)i / (double)(1 << mb)) * ldexp(1.0, e);
            if (v >= HIF8_OVERFLOW_TIE) continue;
            g_positive[n].value = v;
            g_positive[n++].code = (uint8_t)normal_code(e, i);
        }
    }
    qsort(g_positive, (size_t)n, sizeof(hif8o_entry), cmp_entry);
    g_positive_ready = 1;
}

static uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* codec.py:148-180 -- nearest, ties away from zero; under/overflow ties. */
static uint8_t encode_double(double value);

uint8_t hif8o_encode_value(float value_f) { return encode_double((double)value_f); }

static uint8_t encode_double(double value) {
    build_positive();
    if (isnan(value)) return HIF8_NAN;
    if (isinf(value)) return value < 0.0 ? HIF8_NINF : HIF8_PINF;
    double magnitude = fabs(value);
    if (magnitude < HIF8_UNDERFLOW_TIE) return 0x00;
    if (magnitude >= HIF8_OVERFLOW_TIE) return value < 0.0 ? HIF8_NINF : HIF8_PINF;
    /* bisect_left: first index whose value is >= magnitude */
    int lo = 0, hi = 127;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (g_positive[mid].value < magnitude) lo = mid + 1; else hi = mid;
    }
    int upper = lo;
    uint8_t code;
    if (upper == 0) {
        code = g_positive[0].code;
    } else if (upper == 127) {
        code = g_positive[126].code;
    } else {
        int lower = upper - 1;
        double lower_distance = magnitude - g_positive[lower].value;
        double upper_distance = g_positive[upper].value - magnitude;
        code = upper_distance <= lower_distance ? g_positive[upper].code : g_positive[lower].code;
    }
    if (code == 0x00) return code;
    return (uint8_t)(code | (value < 0.0 ? 0x80 : 0x00));
}

/* codec.py:90-103 (decode table) and torch_codec.py:19-29 (encode LUT). */
static void build_tables(void) {
    if (g_tables_ready) return;
    build_positive();
    double positive[128];
    for (int i = 0; i < 128; ++i) positive[i] = NAN;
    for (int i = 0; i < 127; ++i) positive[g_positive[i].code] = g_positive[i].value;
    positive[HIF8_PINF] = INFINITY;
    for (int b = 0; b < 256; ++b) {
        if (b == HIF8_NAN) {
            g_decode[b] = NAN;
            continue;
        }
        double m = positive[b & 0x7F];
        g_decode[b] = (float)((b & 0x80) ? -m : m);
    }
    for (int e = 0; e < 256; ++e)
        for (int t = 0; t < 16; ++t)
            g_lut4096[e * 16 + t] =
                (uint8_t)(hif8o_encode_value(bits_f32(((uint32_t)e << 23) | ((uint32_t)t << 19))) & 0x7F);
    g_tables_ready = 1;
}

float hif8o_decode_value(uint8_t byte) {
    build_tables();
    return g_decode[byte];
}

void hif8o_decode_table(float out[256]) {
    build_tables();
    memcpy(out, g_decode, sizeof(g_decode));
}

void hif8o_encode_lut4096(uint8_t out[4096]) {
    build_tables();
    memcpy(out, g_lut4096, sizeof(g_lut4096));
}

/* codec.py:106-145 -- BF16 payload by field arithmetic. */
uint16_t hif8o_decode_bf16_bits(uint8_t byte) {
    if (byte == HIF8_NAN) return 0x7FC0;
    uint16_t sign = (byte & 0x80) ? 0x8000 : 0;
    int m = byte & 0x7F;
    if (m == 0) return sign;
    if (m == HIF8_PINF) return (uint16_t)(sign | 0x7F80);
    int exponent_field, fraction;
    if (m <= 7) {
        exponent_field = 104 + m;
        fraction = 0;
    } else if (m <= 63) {
        static const int exponent_by_group[8] = {0, 0, 1, -1, 2, 3, -2, -3};
        exponent_field = 127 + exponent_by_group[m >> 3];
        fraction = (m & 0x7) << 4;
    } else if (m <= 79) {
        exponent_field = 131 + ((m - 64) >> 2);
        fraction = (m & 0x3) << 5;
    } else if (m <= 95) {
        exponent_field = 123 - ((m - 80) >> 2);
        fraction = (m & 0x3) << 5;
    } else if (m <= 110) {
        exponent_field = 135 + ((m - 96) >> 1);
        fraction = (m & 0x1) << 6;
    } else {
        exponent_field = 119 - ((m - 112) >> 1);
        fraction = (m & 0x1) << 6;
    }
    return (uint16_t)(sign | (exponent_field << 7) | fraction);
}

/* torch_codec.py:32-49 */
static uint8_t encode_lut_one(float v) {
    uint32_t bits = f32_bits(v);
    uint32_t exponent = (bits >> 23) & 0xFF;
    uint32_t mantissa = bits & 0x007FFFFF;
    uint8_t sign = (uint8_t)((bits >> 24) & 0x80);
    if (exponent == 0xFF) return mantissa != 0 ? HIF8_NAN : (uint8_t)(sign | HIF8_PINF);
    uint8_t magnitude = g_lut4096[exponent * 16 + (mantissa >> 19)];
    return magnitude == 0 ? magnitude : (uint8_t)(magnitude | sign);
}

void hif8o_encode_tensor(const float *x, int64_t n, uint8_t *out) {
    build_tables();
    for (int64_t i = 0; i < n; ++i) out[i] = encode_lut_one(x[i]);
}

float hif8o_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1F;
    uint32_t f = h & 0x3FF;
    if (e == 0) {
        /* zero or subnormal: value = f * 2^-24 (exact in FP32) */
        float v = (float)f * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) return bits_f32(sign | 0x7F800000u | (f << 13));
    return bits_f32(sign | ((e + 112) << 23) | (f << 13));
}

float hif8o_bf16_bits_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

uint16_t hif8o_f32_to_bf16_bits(float v) {
    if (isnan(v)) return 0x7FC0;
    uint32_t u = f32_bits(v);
    uint32_t rounding_bias = 0x7FFF + ((u >> 16) & 1);
    return (uint16_t)((u + rounding_bias) >> 16);
}

uint16_t hif8o_f32_to_f16_bits(float v) {
    uint32_t u = f32_bits(v);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000);
    uint32_t a = u & 0x7FFFFFFF;
    if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00);
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00); /* rounds past 65504 */
    if (a < 0x33000001u) return sign;                        /* below half of 2^-24 */
    int e = (int)(a >> 23) - 127;
    uint32_t mant = (a & 0x7FFFFF) | 0x800000;
    if (e < -14) {
        /* subnormal: value = mant * 2^(e-23) = (mant >> (-e-1)) * 2^-24 */
        int shift = -e - 1;
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q += 1;
        return (uint16_t)(sign | q);
    }
    uint32_t q = mant >> 13;
    uint32_t rem = mant & 0x1FFF;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q += 1;
    uint32_t bits = ((uint32_t)(e + 15) << 10) + (q - 0x400);
    if (q == 0x800) bits = ((uint32_t)(e + 16) << 10);
    return (uint16_t)(sign | bits);
}

static float load_half(const uint16_t *x, int dtype, int64_t i) {
    return dtype == 1 ? hif8o_bf16_bits_to_f32(x[i]) : hif8o_f16_bits_to_f32(x[i]);
}

/* calibration.py:139-158 (saturating encode) + :182-201 (static quant). */
static uint8_t static_encode(float x, float scale) {
    volatile float q = x / scale; /* IEEE single division */
    float v = q;
    if (isfinite(v)) {
        if (v > (float)HIF8_MAX_FINITE) v = (float)HIF8_MAX_FINITE;
        if (v < -(float)HIF8_MAX_FINITE) v = -(float)HIF8_MAX_FINITE;
    }
    return encode_lut_one(v);
}

void hif8o_static_quant(const uint16_t *x, int x_dtype, int64_t rows, int64_t k,
                        const float *scale, int64_t scale_count, uint8_t *out,
                        float *row_scale) {
    build_tables();
    for (int64_t r = 0; r < rows; ++r) {
        float s = scale[r % scale_count];
        if (row_scale) row_scale[r] = s;
        for (int64_t c = 0; c < k; ++c) out[r * k + c] = static_encode(load_half(x, x_dtype, r * k + c), s);
    }
}

/* codec.py:205-255 (choose_row_scale + quantize_rows, scale_factor 1):
 * per row, scale = max(amax of the finite |x|, 1e-12) and every code is
 * encode_ascend(x / scale) with the quotient in double precision, as the
 * Python reference divides Python floats.  NaN / Inf keep their codes. */
void hif8o_dynamic_quant(const uint16_t *x, int x_dtype, int64_t rows, int64_t k, uint8_t *out,
                         float *row_scale) {
    for (int64_t r = 0; r < rows; ++r) {
        double amax = 0.0;
        for (int64_t c = 0; c < k; ++c) {
            const double v = (double)load_half(x, x_dtype, r * k + c);
            if (isfinite(v) && fabs(v) > amax) amax = fabs(v);
        }
        const double scale = amax > 1.0e-12 ? amax : 1.0e-12;
        if (row_scale) row_scale[r] = (float)scale;
        for (int64_t c = 0; c < k; ++c) out[r * k + c] = encode_double((double)load_half(x, x_dtype, r * k + c) / scale);
    }
}

/* tests/test_npu_ops.py:105-123 expectation: (lut[codes] * scale).to(bf16). */
void hif8o_scaled_decode(const uint8_t *data, int64_t rows, int64_t k, int64_t row_stride,
                         const float *scale, uint16_t *out) {
    build_tables();
    for (int64_t r = 0; r < rows; ++r) {
        float s = scale[r];
        for (int64_t c = 0; c < k; ++c) {
            volatile float v = g_decode[data[r * row_stride + c]] * s;
            out[r * k + c] = hif8o_f32_to_bf16_bits(v);
        }
    }
}

/* kv_runtime.py:1168-1199 (_quantize_kv), kv_cache.py:151-170 (pack_kv_rows),
 * kv_runtime.py:1296-1316 (slot mapping, index_copy_). */
int64_t hif8o_kv_write(const uint16_t *src, int src_dtype, int64_t tokens, int64_t heads,
                       int64_t head_size, const float *head_scale, const int64_t *slot_mapping,
                       uint8_t *cache, int64_t num_blocks, int64_t block_size) {
    build_tables();
    int64_t rejected = 0;
    const int64_t width = head_size + 4;
    for (int64_t t = 0; t < tokens; ++t) {
        int64_t slot = slot_mapping[t];
        if (slot < 0) continue;
        int64_t block = slot / block_size;
        int64_t offset = slot % block_size;
        if (block >= num_blocks) {
            ++rejected;
            continue;
        }
        for (int64_t h = 0; h < heads; ++h) {
            uint8_t *row = cache + ((block * block_size + offset) * heads + h) * width;
            float s = head_scale[h];
            for (int64_t c = 0; c < head_size; ++c)
                row[c] = static_encode(load_half(src, src_dtype, (t * heads + h) * head_size + c), s);
            memcpy(row + head_size, &s, 4); /* little-endian FP32 sidecar */
        }
    }
    return rejected;
}

/* reference.py:10-43 */
void hif8o_linear_f64(const uint8_t *a, const uint8_t *w, const float *a_scale,
                      const float *w_scale, const float *bias, int64_t m, int64_t n,
                      int64_t k, double *out) {
    build_tables();
    for (int64_t i = 0; i < m; ++i) {
        for (int64_t j = 0; j < n; ++j) {
            double acc = 0.0;
            for (int64_t c = 0; c < k; ++c)
                acc += (double)g_decode[a[i * k + c]] * (double)g_decode[w[j * k + c]];
            double value = acc * (double)a_scale[i] * (double)w_scale[j];
            if (bias) value += (double)bias[j];
            out[i * n + j] = value;
        }
    }
}
