/*
 * gemm_oracle.c -- CPU restatement of slang-gemm's scalar reference GEMMs
 * (src/gemm.zig). TEST INFRASTRUCTURE ONLY: the product library never links
 * or calls this file; tests/, the smoke check and bench.py's CPU legs load it
 * as the checker / CPU baseline.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, so that every f32/f64
 * multiply and add rounds separately, as Zig's default strict float mode does).
 */
#include "gemm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* Layout helpers                                                             */
/* ------------------------------------------------------------------------- */

/* matrixLayout (src/gemm.zig:165-170) */
or_layout or_matrix_layout(int layout, size_t ld) {
    or_layout l;
    l.offset = 0;
    if (layout == OR_ROW_MAJOR) { l.row_stride = ld; l.col_stride = 1; }
    else { l.row_stride = 1; l.col_stride = ld; }
    return l;
}

/* storedRows / storedCols (src/gemm.zig:172-184) */
size_t or_stored_rows(int op, size_t rows, size_t cols) { return op == OR_OP_N ? rows : cols; }
size_t or_stored_cols(int op, size_t rows, size_t cols) { return op == OR_OP_N ? cols : rows; }

/* minimumLd (src/gemm.zig:186-191) */
size_t or_minimum_ld(int layout, size_t rows, size_t cols) {
    size_t v = layout == OR_ROW_MAJOR ? cols : rows;
    return v > 1 ? v : 1;
}

static inline size_t lidx(or_layout l, size_t r, size_t c) { return l.offset + r * l.row_stride + c * l.col_stride; }

/* matrixExtent (src/gemm.zig:708-711) */
size_t or_matrix_extent(or_layout l, size_t rows, size_t cols) {
    if (rows == 0 || cols == 0) return 0;
    return lidx(l, rows - 1, cols - 1) + 1;
}

/* elementSize (src/gemm.zig:777-788) */
size_t or_element_size(int t) {
    switch (t) {
    case OR_R_16F: case OR_R_16BF: case OR_R_16I: case OR_R_16U: return 2;
    case OR_C_16F: case OR_C_16BF: case OR_C_16I: case OR_C_16U: return 4;
    case OR_R_32F: case OR_R_32I: case OR_R_32U: return 4;
    case OR_C_32F: case OR_C_32I: case OR_C_32U: return 8;
    case OR_R_64F: case OR_R_64I: case OR_R_64U: return 8;
    case OR_C_64F: case OR_C_64I: case OR_C_64U: return 16;
    case OR_R_4I: case OR_R_4U: case OR_R_8I: case OR_R_8U: case OR_R_8F_E4M3: case OR_R_8F_E5M2:
    case OR_R_8F_UE8M0: case OR_R_6F_E2M3: case OR_R_6F_E3M2: case OR_R_4F_E2M1: return 1;
    case OR_C_4I: case OR_C_4U: case OR_C_8I: case OR_C_8U: return 2;
    default: return 0;
    }
}

/* isComplexType (src/gemm.zig:790-795) */
int or_is_complex_type(int t) {
    switch (t) {
    case OR_C_16F: case OR_C_16BF: case OR_C_32F: case OR_C_64F: case OR_C_4I: case OR_C_4U: case OR_C_8I:
    case OR_C_8U: case OR_C_16I: case OR_C_16U: case OR_C_32I: case OR_C_32U: case OR_C_64I: case OR_C_64U:
        return 1;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------- */
/* Codecs (src/gemm.zig:914-1010)                                             */
/* ------------------------------------------------------------------------- */

static inline uint32_t f32_bits(float v) { uint32_t x; memcpy(&x, &v, 4); return x; }
static inline float bits_f32(uint32_t x) { float v; memcpy(&v, &x, 4); return v; }

/* f32ToF16Bits (src/gemm.zig:914-917): Zig's @floatCast(f32 -> f16), i.e. IEEE
 * round-to-nearest-even, overflow to infinity, gradual underflow. Written out
 * on the bit pattern. */
uint16_t or_f32_to_f16_bits(float v) {
    uint32_t x = f32_bits(v);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7c00u | 0x200u | (man >> 13)); /* quiet NaN, keep top payload */
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e >= 1) {
        uint32_t val = ((uint32_t)e << 10) | (man >> 13);
        uint32_t rem = man & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (val & 1u))) val++;
        if (val >= 0x7c00u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | val);
    }
    if (e < -10) return (uint16_t)sign;
    /* f16 subnormal: value = val * 2^-24 */
    uint32_t sig = man | 0x800000u;
    int shift = 14 - e; /* 14..24 */
    uint32_t val = sig >> shift;
    uint32_t rem = sig & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (val & 1u))) val++;
    return (uint16_t)(sign | val);
}

/* f16BitsToF32 (src/gemm.zig:919-922): exact widening. */
float or_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        float mag = ldexpf((float)m, -24);
        return sign ? -mag : mag;
    }
    if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
    return bits_f32(sign | ((e - 15u + 127u) << 23) | (m << 13));
}

/* f32ToBf16Bits (src/gemm.zig:924-928): raw + 0x7fff + lsb, truncated (no NaN case). */
uint16_t or_f32_to_bf16_bits(float v) {
    uint32_t raw = f32_bits(v);
    uint32_t rounded = raw + 0x7fffu + ((raw >> 16) & 1u);
    return (uint16_t)(rounded >> 16);
}

/* bf16BitsToF32 (src/gemm.zig:930-933) */
float or_bf16_bits_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

/* tinyFloatToF32 (src/gemm.zig:943-962) */
static float tiny_float_to_f32(uint8_t bits, int exp_bits, int mant_bits, int bias) {
    int sign = (bits >> (exp_bits + mant_bits)) & 1;
    uint8_t exp_mask = (uint8_t)((1u << exp_bits) - 1u);
    uint8_t mant_mask = (uint8_t)((1u << mant_bits) - 1u);
    int exp_raw = (bits >> mant_bits) & exp_mask;
    int mant_raw = bits & mant_mask;
    float sign_scale = sign == 0 ? 1.0f : -1.0f;
    if (exp_raw == 0 && mant_raw == 0) return sign == 0 ? 0.0f : -0.0f;
    float mant_den = (float)(1u << mant_bits);
    if (exp_raw == 0) {
        int exponent = 1 - bias;
        return sign_scale * ((float)mant_raw / mant_den) * ldexpf(1.0f, exponent);
    }
    int exponent = exp_raw - bias;
    float mant = 1.0f + (float)mant_raw / mant_den;
    return sign_scale * mant * ldexpf(1.0f, exponent);
}

float or_fp8_e4m3_to_f32(uint8_t bits) { return tiny_float_to_f32(bits, 4, 3, 7); }
float or_fp8_e5m2_to_f32(uint8_t bits) { return tiny_float_to_f32(bits, 5, 2, 15); }

static inline uint16_t rd16(const uint8_t *d, size_t o) { return (uint16_t)(d[o] | (d[o + 1] << 8)); }
static inline uint32_t rd32(const uint8_t *d, size_t o) { uint32_t v; memcpy(&v, d + o, 4); return v; }
static inline uint64_t rd64(const uint8_t *d, size_t o) { uint64_t v; memcpy(&v, d + o, 8); return v; }
static inline void wr16(uint8_t *d, size_t o, uint16_t v) { d[o] = (uint8_t)v; d[o + 1] = (uint8_t)(v >> 8); }
static inline void wr32(uint8_t *d, size_t o, uint32_t v) { memcpy(d + o, &v, 4); }
static inline void wr64(uint8_t *d, size_t o, uint64_t v) { memcpy(d + o, &v, 8); }
static inline double rdf32(const uint8_t *d, size_t o) { return (double)bits_f32(rd32(d, o)); }
static inline double rdf64(const uint8_t *d, size_t o) { double v; uint64_t x = rd64(d, o); memcpy(&v, &x, 8); return v; }
static inline int8_t sign_extend4(uint8_t v) { uint8_t low = v & 0x0f; return (low & 0x08) == 0 ? (int8_t)low : (int8_t)((int)low - 16); }

/* readScalar (src/gemm.zig:797-835) */
void or_read_scalar(const uint8_t *d, int t, size_t index, or_scalar *out) {
    size_t o = index * or_element_size(t);
    double re = 0.0, im = 0.0;
    switch (t) {
    case OR_R_16F: re = or_f16_bits_to_f32(rd16(d, o)); break;
    case OR_C_16F: re = or_f16_bits_to_f32(rd16(d, o)); im = or_f16_bits_to_f32(rd16(d, o + 2)); break;
    case OR_R_16BF: re = or_bf16_bits_to_f32(rd16(d, o)); break;
    case OR_C_16BF: re = or_bf16_bits_to_f32(rd16(d, o)); im = or_bf16_bits_to_f32(rd16(d, o + 2)); break;
    case OR_R_32F: re = rdf32(d, o); break;
    case OR_C_32F: re = rdf32(d, o); im = rdf32(d, o + 4); break;
    case OR_R_64F: re = rdf64(d, o); break;
    case OR_C_64F: re = rdf64(d, o); im = rdf64(d, o + 8); break;
    case OR_R_4I: re = sign_extend4(d[o] & 0x0f); break;
    case OR_C_4I: re = sign_extend4(d[o] & 0x0f); im = sign_extend4(d[o + 1] & 0x0f); break;
    case OR_R_4U: re = d[o] & 0x0f; break;
    case OR_C_4U: re = d[o] & 0x0f; im = d[o + 1] & 0x0f; break;
    case OR_R_8I: re = (int8_t)d[o]; break;
    case OR_C_8I: re = (int8_t)d[o]; im = (int8_t)d[o + 1]; break;
    case OR_R_8U: re = d[o]; break;
    case OR_C_8U: re = d[o]; im = d[o + 1]; break;
    case OR_R_16I: re = (int16_t)rd16(d, o); break;
    case OR_C_16I: re = (int16_t)rd16(d, o); im = (int16_t)rd16(d, o + 2); break;
    case OR_R_16U: re = rd16(d, o); break;
    case OR_C_16U: re = rd16(d, o); im = rd16(d, o + 2); break;
    case OR_R_32I: re = (int32_t)rd32(d, o); break;
    case OR_C_32I: re = (int32_t)rd32(d, o); im = (int32_t)rd32(d, o + 4); break;
    case OR_R_32U: re = rd32(d, o); break;
    case OR_C_32U: re = rd32(d, o); im = rd32(d, o + 4); break;
    case OR_R_64I: re = (double)(int64_t)rd64(d, o); break;
    case OR_C_64I: re = (double)(int64_t)rd64(d, o); im = (double)(int64_t)rd64(d, o + 8); break;
    case OR_R_64U: re = (double)rd64(d, o); break;
    case OR_C_64U: re = (double)rd64(d, o); im = (double)rd64(d, o + 8); break;
    case OR_R_8F_E4M3: re = or_fp8_e4m3_to_f32(d[o]); break;
    case OR_R_8F_E5M2: re = or_fp8_e5m2_to_f32(d[o]); break;
    case OR_R_8F_UE8M0: re = ldexpf(1.0f, (int)d[o] - 127); break;
    case OR_R_6F_E2M3: re = tiny_float_to_f32(d[o] & 0x3f, 2, 3, 1); break;
    case OR_R_6F_E3M2: re = tiny_float_to_f32(d[o] & 0x3f, 3, 2, 3); break;
    case OR_R_4F_E2M1: re = tiny_float_to_f32(d[o] & 0x0f, 2, 1, 1); break;
    default: break;
    }
    out->re = re;
    out->im = im;
}

/* clampInt (src/gemm.zig:1002-1010): round half away from zero, clamp, convert.
 * fmin/fmax return the non-NaN operand, like Zig's @min/@max. */
static int64_t clamp_int(int bits, double v) {
    double lo = -ldexp(1.0, bits - 1);
    double hi = ldexp(1.0, bits - 1) - 1.0;
    double r = fmin(hi, fmax(lo, round(v)));
    if (r >= 9223372036854775807.0) return INT64_MAX;
    return (int64_t)r;
}

/* clampUnsigned (src/gemm.zig:1012-1016) */
static uint64_t clamp_unsigned(int bits, double v) {
    double hi = ldexp(1.0, bits) - 1.0;
    double r = fmin(hi, fmax(0.0, round(v)));
    if (r >= 18446744073709551615.0) return UINT64_MAX;
    return (uint64_t)r;
}

/* quantizeByte (src/gemm.zig:986-995) */
static uint8_t quantize_byte(int t, double v) {
    switch (t) {
    case OR_R_4I: return (uint8_t)((int8_t)clamp_int(4, v)) & 0x0f;
    case OR_R_4U: {
        double r = fmax(0.0, round(v));
        uint64_t u = r >= 18446744073709551615.0 ? UINT64_MAX : (uint64_t)r;
        return (uint8_t)(u < 15 ? u : 15);
    }
    case OR_R_8I: return (uint8_t)(int8_t)clamp_int(8, v);
    default: return (uint8_t)clamp_unsigned(8, v);
    }
}

static int component_type(int t) {
    switch (t) {
    case OR_C_4I: return OR_R_4I;
    case OR_C_4U: return OR_R_4U;
    case OR_C_8I: return OR_R_8I;
    case OR_C_8U: return OR_R_8U;
    default: return t;
    }
}

static inline void wrf32(uint8_t *d, size_t o, double v) { wr32(d, o, f32_bits((float)v)); }
static inline void wrf64(uint8_t *d, size_t o, double v) { uint64_t x; memcpy(&x, &v, 8); wr64(d, o, x); }

/* writeScalar (src/gemm.zig:837-896). Note the double rounding f64 -> f32 -> f16/bf16. */
void or_write_scalar(uint8_t *d, int t, size_t index, const or_scalar *v) {
    size_t o = index * or_element_size(t);
    switch (t) {
    case OR_R_16F: wr16(d, o, or_f32_to_f16_bits((float)v->re)); break;
    case OR_C_16F: wr16(d, o, or_f32_to_f16_bits((float)v->re)); wr16(d, o + 2, or_f32_to_f16_bits((float)v->im)); break;
    case OR_R_16BF: wr16(d, o, or_f32_to_bf16_bits((float)v->re)); break;
    case OR_C_16BF: wr16(d, o, or_f32_to_bf16_bits((float)v->re)); wr16(d, o + 2, or_f32_to_bf16_bits((float)v->im)); break;
    case OR_R_32F: wrf32(d, o, v->re); break;
    case OR_C_32F: wrf32(d, o, v->re); wrf32(d, o + 4, v->im); break;
    case OR_R_64F: wrf64(d, o, v->re); break;
    case OR_C_64F: wrf64(d, o, v->re); wrf64(d, o + 8, v->im); break;
    case OR_R_4I: case OR_R_4U: case OR_R_8I: case OR_R_8U: case OR_R_8F_E4M3: case OR_R_8F_E5M2:
    case OR_R_8F_UE8M0: case OR_R_6F_E2M3: case OR_R_6F_E3M2: case OR_R_4F_E2M1:
        d[o] = quantize_byte(t, v->re); break;
    case OR_C_4I: case OR_C_4U: case OR_C_8I: case OR_C_8U:
        d[o] = quantize_byte(component_type(t), v->re);
        d[o + 1] = quantize_byte(component_type(t), v->im);
        break;
    case OR_R_16I: wr16(d, o, (uint16_t)(int16_t)clamp_int(16, v->re)); break;
    case OR_C_16I: wr16(d, o, (uint16_t)(int16_t)clamp_int(16, v->re)); wr16(d, o + 2, (uint16_t)(int16_t)clamp_int(16, v->im)); break;
    case OR_R_16U: wr16(d, o, (uint16_t)clamp_unsigned(16, v->re)); break;
    case OR_C_16U: wr16(d, o, (uint16_t)clamp_unsigned(16, v->re)); wr16(d, o + 2, (uint16_t)clamp_unsigned(16, v->im)); break;
    case OR_R_32I: wr32(d, o, (uint32_t)(int32_t)clamp_int(32, v->re)); break;
    case OR_C_32I: wr32(d, o, (uint32_t)(int32_t)clamp_int(32, v->re)); wr32(d, o + 4, (uint32_t)(int32_t)clamp_int(32, v->im)); break;
    case OR_R_32U: wr32(d, o, (uint32_t)clamp_unsigned(32, v->re)); break;
    case OR_C_32U: wr32(d, o, (uint32_t)clamp_unsigned(32, v->re)); wr32(d, o + 4, (uint32_t)clamp_unsigned(32, v->im)); break;
    case OR_R_64I: wr64(d, o, (uint64_t)clamp_int(64, v->re)); break;
    case OR_C_64I: wr64(d, o, (uint64_t)clamp_int(64, v->re)); wr64(d, o + 8, (uint64_t)clamp_int(64, v->im)); break;
    case OR_R_64U: wr64(d, o, clamp_unsigned(64, v->re)); break;
    case OR_C_64U: wr64(d, o, clamp_unsigned(64, v->re)); wr64(d, o + 8, clamp_unsigned(64, v->im)); break;
    default: break;
    }
}

/* ------------------------------------------------------------------------- */
/* Validation (src/gemm.zig:713-775)                                          */
/* ------------------------------------------------------------------------- */

/* validateSliceLen (src/gemm.zig:733-739) */
static int validate_slice_len(size_t len, size_t extent, size_t stride, size_t batch_count) {
    if (extent == 0) return OR_OK;
    size_t used = stride == 0 ? extent : stride;
    if (used < extent) return OR_ERR_INVALID_STRIDE;
    size_t required = (batch_count - 1) * used + extent;
    if (len < required) return OR_ERR_BUFFER_TOO_SMALL;
    return OR_OK;
}

/* validateByteSliceLen (src/gemm.zig:769-775): `stride` is already resolved. */
static int validate_byte_slice_len(size_t len, int t, size_t extent, size_t stride, size_t batch_count) {
    if (extent == 0) return OR_OK;
    if (stride < extent) return OR_ERR_INVALID_STRIDE;
    size_t required = ((batch_count - 1) * stride + extent) * or_element_size(t);
    if (len < required) return OR_ERR_BUFFER_TOO_SMALL;
    return OR_OK;
}

/* ------------------------------------------------------------------------- */
/* gemm(f32) (src/gemm.zig:523-544)                                           */
/* ------------------------------------------------------------------------- */

typedef struct f32_job {
    int op_a, op_b;
    size_t m, n, k;
    float alpha, beta;
    const float *a, *b;
    float *c;
    or_layout al, bl, cl;
    size_t sa, sb, sc;
} f32_job;

/* loadOp (src/gemm.zig:745-751); conj is the identity for real T. */
static inline float load_op_f32(const float *d, or_layout l, int op, size_t base, size_t r, size_t c) {
    return op == OR_OP_N ? d[base + lidx(l, r, c)] : d[base + lidx(l, c, r)];
}

/* One output element, in the reference's order: sum_k in f32, then
 * alpha*sum + beta*c with each product rounded to f32. */
static void f32_cols(const f32_job *j, size_t batch, size_t col_begin, size_t col_end) {
    size_t a_base = batch * j->sa, b_base = batch * j->sb, c_base = batch * j->sc;
    for (size_t row = 0; row < j->m; ++row) {
        for (size_t col = col_begin; col < col_end; ++col) {
            float sum = 0.0f;
            for (size_t kk = 0; kk < j->k; ++kk) {
                float prod = load_op_f32(j->a, j->al, j->op_a, a_base, row, kk) *
                             load_op_f32(j->b, j->bl, j->op_b, b_base, kk, col);
                sum = sum + prod;
            }
            size_t ci = c_base + lidx(j->cl, row, col);
            float t1 = j->alpha * sum;
            float t2 = j->beta * j->c[ci];
            j->c[ci] = t1 + t2;
        }
    }
}

/* Parallel driver: the flattened (batch, col) space is cut into contiguous
 * ranges, one per thread. Per-element arithmetic is untouched. */
typedef void (*range_fn)(const void *job, size_t batch, size_t col_begin, size_t col_end);

typedef struct range_task {
    range_fn fn;
    const void *job;
    size_t n;       /* columns per batch */
    size_t begin;   /* flattened (batch*n + col) range */
    size_t end;
} range_task;

static void *range_worker(void *arg) {
    range_task *t = (range_task *)arg;
    size_t i = t->begin;
    while (i < t->end) {
        size_t batch = i / t->n, col = i % t->n;
        size_t stop = (batch + 1) * t->n;
        if (stop > t->end) stop = t->end;
        t->fn(t->job, batch, col, col + (stop - i));
        i = stop;
    }
    return NULL;
}

static void run_ranges(range_fn fn, const void *job, size_t batch_count, size_t n, int threads) {
    size_t total = batch_count * n;
    if (total == 0) return;
    if (threads < 1) threads = 1;
    if ((size_t)threads > total) threads = (int)total;
    range_task *tasks = (range_task *)calloc((size_t)threads, sizeof(range_task));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int *started = (int *)calloc((size_t)threads, sizeof(int));
    for (int t = 0; t < threads; ++t) {
        tasks[t].fn = fn;
        tasks[t].job = job;
        tasks[t].n = n;
        tasks[t].begin = total * (size_t)t / (size_t)threads;
        tasks[t].end = total * (size_t)(t + 1) / (size_t)threads;
        if (t > 0) started[t] = pthread_create(&tids[t], NULL, range_worker, &tasks[t]) == 0;
    }
    range_worker(&tasks[0]);
    for (int t = 1; t < threads; ++t) {
        if (started[t]) pthread_join(tids[t], NULL);
        else range_worker(&tasks[t]); /* thread creation failed: do the range here */
    }
    free(started);
    free(tids);
    free(tasks);
}

static void f32_range(const void *job, size_t batch, size_t cb, size_t ce) { f32_cols((const f32_job *)job, batch, cb, ce); }

static int gemm_f32_impl(int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                         const float *a, size_t a_len, or_layout al,
                         const float *b, size_t b_len, or_layout bl, float beta,
                         float *c, size_t c_len, or_layout cl,
                         size_t batch_count, size_t stride_a, size_t stride_b, size_t stride_c, int threads) {
    /* validateScalarDesc (src/gemm.zig:713-721) */
    if (batch_count == 0) return OR_ERR_INVALID_BATCH_COUNT;
    size_t a_ext = or_matrix_extent(al, or_stored_rows(op_a, m, k), or_stored_cols(op_a, m, k));
    size_t b_ext = or_matrix_extent(bl, or_stored_rows(op_b, k, n), or_stored_cols(op_b, k, n));
    size_t c_ext = or_matrix_extent(cl, m, n);
    int rc;
    if ((rc = validate_slice_len(a_len, a_ext, stride_a, batch_count))) return rc;
    if ((rc = validate_slice_len(b_len, b_ext, stride_b, batch_count))) return rc;
    if ((rc = validate_slice_len(c_len, c_ext, stride_c, batch_count))) return rc;
    f32_job j;
    j.op_a = op_a; j.op_b = op_b; j.m = m; j.n = n; j.k = k; j.alpha = alpha; j.beta = beta;
    j.a = a; j.b = b; j.c = c; j.al = al; j.bl = bl; j.cl = cl;
    j.sa = stride_a == 0 ? a_ext : stride_a;
    j.sb = stride_b == 0 ? b_ext : stride_b;
    j.sc = stride_c == 0 ? c_ext : stride_c;
    if (threads <= 1) {
        for (size_t batch = 0; batch < batch_count; ++batch) f32_cols(&j, batch, 0, n);
    } else {
        run_ranges(f32_range, &j, batch_count, n, threads);
    }
    return OR_OK;
}

int or_gemm_f32(int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                const float *a, size_t a_len, or_layout al,
                const float *b, size_t b_len, or_layout bl, float beta,
                float *c, size_t c_len, or_layout cl,
                size_t batch_count, size_t stride_a, size_t stride_b, size_t stride_c) {
    return gemm_f32_impl(op_a, op_b, m, n, k, alpha, a, a_len, al, b, b_len, bl, beta, c, c_len, cl,
                         batch_count, stride_a, stride_b, stride_c, 1);
}

int or_sgemm(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
             const float *a, size_t a_len, size_t lda, const float *b, size_t b_len, size_t ldb,
             float beta, float *c, size_t c_len, size_t ldc) {
    return gemm_f32_impl(op_a, op_b, m, n, k, alpha, a, a_len, or_matrix_layout(layout, lda), b, b_len,
                         or_matrix_layout(layout, ldb), beta, c, c_len, or_matrix_layout(layout, ldc), 1, 0, 0, 0, 1);
}

int or_sgemm_strided_batched(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                             const float *a, size_t a_len, size_t lda, size_t stride_a,
                             const float *b, size_t b_len, size_t ldb, size_t stride_b, float beta,
                             float *c, size_t c_len, size_t ldc, size_t stride_c, size_t batch_count) {
    return gemm_f32_impl(op_a, op_b, m, n, k, alpha, a, a_len, or_matrix_layout(layout, lda), b, b_len,
                         or_matrix_layout(layout, ldb), beta, c, c_len, or_matrix_layout(layout, ldc),
                         batch_count, stride_a, stride_b, stride_c, 1);
}

int or_sgemm_strided_batched_mt(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                                const float *a, size_t a_len, size_t lda, size_t stride_a,
                                const float *b, size_t b_len, size_t ldb, size_t stride_b, float beta,
                                float *c, size_t c_len, size_t ldc, size_t stride_c, size_t batch_count,
                                int threads) {
    return gemm_f32_impl(op_a, op_b, m, n, k, alpha, a, a_len, or_matrix_layout(layout, lda), b, b_len,
                         or_matrix_layout(layout, ldb), beta, c, c_len, or_matrix_layout(layout, ldc),
                         batch_count, stride_a, stride_b, stride_c, threads);
}

/* ------------------------------------------------------------------------- */
/* hgemm (src/gemm.zig:438-477)                                               */
/* ------------------------------------------------------------------------- */

int or_hgemm(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, uint16_t alpha,
             const uint16_t *a, size_t lda, const uint16_t *b, size_t ldb, uint16_t beta,
             uint16_t *c, size_t ldc) {
    or_layout al = or_matrix_layout(layout, lda), bl = or_matrix_layout(layout, ldb), cl = or_matrix_layout(layout, ldc);
    float alpha_f = or_f16_bits_to_f32(alpha), beta_f = or_f16_bits_to_f32(beta);
    for (size_t row = 0; row < m; ++row) {
        for (size_t col = 0; col < n; ++col) {
            float sum = 0.0f;
            for (size_t kk = 0; kk < k; ++kk) {
                float av = op_a == OR_OP_N ? or_f16_bits_to_f32(a[lidx(al, row, kk)]) : or_f16_bits_to_f32(a[lidx(al, kk, row)]);
                float bv = op_b == OR_OP_N ? or_f16_bits_to_f32(b[lidx(bl, kk, col)]) : or_f16_bits_to_f32(b[lidx(bl, col, kk)]);
                float prod = av * bv;
                sum = sum + prod;
            }
            size_t ci = lidx(cl, row, col);
            float t1 = alpha_f * sum;
            float t2 = beta_f * or_f16_bits_to_f32(c[ci]);
            c[ci] = or_f32_to_f16_bits(t1 + t2);
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------------------- */
/* gemmExLegacy (src/gemm.zig:608-630)                                        */
/* ------------------------------------------------------------------------- */

int or_gemm_ex_legacy(int bf16_input, int op_a, int op_b, size_t m, size_t n, size_t k,
                      const uint16_t *a, size_t a_len, or_layout al,
                      const uint16_t *b, size_t b_len, or_layout bl,
                      float *c, size_t c_len, or_layout cl, float alpha, float beta,
                      size_t batch_count, size_t stride_a, size_t stride_b, size_t stride_c) {
    if (batch_count == 0) return OR_ERR_INVALID_BATCH_COUNT;
    size_t a_ext = or_matrix_extent(al, or_stored_rows(op_a, m, k), or_stored_cols(op_a, m, k));
    size_t b_ext = or_matrix_extent(bl, or_stored_rows(op_b, k, n), or_stored_cols(op_b, k, n));
    size_t c_ext = or_matrix_extent(cl, m, n);
    int rc;
    if ((rc = validate_slice_len(a_len, a_ext, stride_a, batch_count))) return rc;
    if ((rc = validate_slice_len(b_len, b_ext, stride_b, batch_count))) return rc;
    if ((rc = validate_slice_len(c_len, c_ext, stride_c, batch_count))) return rc;
    size_t sa = stride_a ? stride_a : a_ext, sb = stride_b ? stride_b : b_ext, sc = stride_c ? stride_c : c_ext;
    for (size_t batch = 0; batch < batch_count; ++batch) {
        for (size_t row = 0; row < m; ++row) {
            for (size_t col = 0; col < n; ++col) {
                float sum = 0.0f;
                for (size_t kk = 0; kk < k; ++kk) {
                    uint16_t ab = op_a == OR_OP_N ? a[batch * sa + lidx(al, row, kk)] : a[batch * sa + lidx(al, kk, row)];
                    uint16_t bb = op_b == OR_OP_N ? b[batch * sb + lidx(bl, kk, col)] : b[batch * sb + lidx(bl, col, kk)];
                    float av = bf16_input ? or_bf16_bits_to_f32(ab) : or_f16_bits_to_f32(ab);
                    float bv = bf16_input ? or_bf16_bits_to_f32(bb) : or_f16_bits_to_f32(bb);
                    float prod = av * bv;
                    sum = sum + prod;
                }
                size_t ci = batch * sc + lidx(cl, row, col);
                float t1 = alpha * sum;
                float t2 = beta * c[ci];
                c[ci] = t1 + t2;
            }
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------------------- */
/* gemmExCuda (src/gemm.zig:671-706)                                          */
/* ------------------------------------------------------------------------- */

typedef struct ex_job {
    const or_ex_desc *d;
    or_layout al, bl, cl;
    size_t sa, sb, sc;
} ex_job;

/* scalarAdd / scalarMul / scalarConj (src/gemm.zig:964-974): full complex
 * arithmetic in f64 even for real types, as the reference does. */
static inline or_scalar s_add(or_scalar a, or_scalar b) { or_scalar r; r.re = a.re + b.re; r.im = a.im + b.im; return r; }
static inline or_scalar s_mul(or_scalar a, or_scalar b) {
    or_scalar r;
    double t1 = a.re * b.re, t2 = a.im * b.im, t3 = a.re * b.im, t4 = a.im * b.re;
    r.re = t1 - t2;
    r.im = t3 + t4;
    return r;
}

/* loadExScalar (src/gemm.zig:761-767) */
static inline or_scalar load_ex(const uint8_t *d, int t, or_layout l, int op, size_t base, size_t r, size_t c) {
    or_scalar v;
    if (op == OR_OP_N) or_read_scalar(d, t, base + lidx(l, r, c), &v);
    else or_read_scalar(d, t, base + lidx(l, c, r), &v);
    if (op == OR_OP_C) v.im = -v.im;
    return v;
}

/* Specialised element decoders for the real input types of the hot configs.
 * They produce the same Scalar as or_read_scalar (imaginary part +0.0). */
#define DEC_R_16F(p, i) ((double)or_f16_bits_to_f32(rd16((p), (i) * 2)))
#define DEC_R_16BF(p, i) ((double)or_bf16_bits_to_f32(rd16((p), (i) * 2)))
#define DEC_R_8I(p, i) ((double)(int8_t)(p)[(i)])
#define DEC_R_32F(p, i) (rdf32((p), (i) * 4))

/* sum over k of the complex product, exactly as gemmExCuda's inner loop. */
#define SUM_LOOP(DECA, DECB)                                                          \
    for (size_t kk = 0; kk < kdim; ++kk) {                                            \
        size_t ia = op_a == OR_OP_N ? a_base + lidx(al, row, kk) : a_base + lidx(al, kk, row); \
        size_t ib = op_b == OR_OP_N ? b_base + lidx(bl, kk, col) : b_base + lidx(bl, col, kk); \
        or_scalar av, bv;                                                             \
        av.re = DECA(a, ia); av.im = 0.0;                                             \
        bv.re = DECB(b, ib); bv.im = 0.0;                                             \
        if (op_a == OR_OP_C) av.im = -av.im;                                          \
        if (op_b == OR_OP_C) bv.im = -bv.im;                                          \
        sum = s_add(sum, s_mul(av, bv));                                              \
    }

static or_scalar ex_sum(const ex_job *j, size_t batch, size_t row, size_t col) {
    const or_ex_desc *d = j->d;
    const uint8_t *a = d->a, *b = d->b;
    or_layout al = j->al, bl = j->bl;
    int op_a = d->op_a, op_b = d->op_b;
    size_t kdim = d->k;
    size_t a_base = batch * j->sa, b_base = batch * j->sb;
    or_scalar sum; sum.re = 0.0; sum.im = 0.0;
    int ta = d->a_type, tb = d->b_type;
    if (ta == OR_R_16F && tb == OR_R_16F) { SUM_LOOP(DEC_R_16F, DEC_R_16F) }
    else if (ta == OR_R_16BF && tb == OR_R_16BF) { SUM_LOOP(DEC_R_16BF, DEC_R_16BF) }
    else if (ta == OR_R_8I && tb == OR_R_8I) { SUM_LOOP(DEC_R_8I, DEC_R_8I) }
    else if (ta == OR_R_32F && tb == OR_R_32F) { SUM_LOOP(DEC_R_32F, DEC_R_32F) }
    else {
        for (size_t kk = 0; kk < kdim; ++kk) {
            or_scalar av = load_ex(a, ta, al, op_a, a_base, row, kk);
            or_scalar bv = load_ex(b, tb, bl, op_b, b_base, kk, col);
            sum = s_add(sum, s_mul(av, bv));
        }
    }
    return sum;
}

static or_scalar ex_final(const or_ex_desc *d, or_scalar sum, const uint8_t *c, size_t ci) {
    or_scalar old;
    or_read_scalar(c, d->c_type, ci, &old);
    return s_add(s_mul(d->alpha, sum), s_mul(d->beta, old));
}

static void ex_cols(const ex_job *j, size_t batch, size_t col_begin, size_t col_end) {
    const or_ex_desc *d = j->d;
    size_t c_base = batch * j->sc;
    for (size_t row = 0; row < d->m; ++row) {
        for (size_t col = col_begin; col < col_end; ++col) {
            or_scalar sum = ex_sum(j, batch, row, col);
            size_t ci = c_base + lidx(j->cl, row, col);
            or_scalar v = ex_final(d, sum, d->c, ci);
            or_write_scalar(d->c, d->c_type, ci, &v);
        }
    }
}

static void ex_range(const void *job, size_t batch, size_t cb, size_t ce) { ex_cols((const ex_job *)job, batch, cb, ce); }

static int ex_prepare(const or_ex_desc *d, ex_job *j) {
    if (d->batch_count == 0) return OR_ERR_INVALID_BATCH_COUNT;
    if (or_element_size(d->a_type) == 0 || or_element_size(d->b_type) == 0 || or_element_size(d->c_type) == 0)
        return OR_ERR_INVALID_TYPE;
    j->d = d;
    j->al = or_matrix_layout(d->layout, d->lda);
    j->bl = or_matrix_layout(d->layout, d->ldb);
    j->cl = or_matrix_layout(d->layout, d->ldc);
    size_t a_ext = or_matrix_extent(j->al, or_stored_rows(d->op_a, d->m, d->k), or_stored_cols(d->op_a, d->m, d->k));
    size_t b_ext = or_matrix_extent(j->bl, or_stored_rows(d->op_b, d->k, d->n), or_stored_cols(d->op_b, d->k, d->n));
    size_t c_ext = or_matrix_extent(j->cl, d->m, d->n);
    j->sa = d->stride_a == 0 ? a_ext : d->stride_a;
    j->sb = d->stride_b == 0 ? b_ext : d->stride_b;
    j->sc = d->stride_c == 0 ? c_ext : d->stride_c;
    int rc;
    if ((rc = validate_byte_slice_len(d->a_len, d->a_type, a_ext, j->sa, d->batch_count))) return rc;
    if ((rc = validate_byte_slice_len(d->b_len, d->b_type, b_ext, j->sb, d->batch_count))) return rc;
    if ((rc = validate_byte_slice_len(d->c_len, d->c_type, c_ext, j->sc, d->batch_count))) return rc;
    return OR_OK;
}

int or_gemm_ex(const or_ex_desc *d) {
    ex_job j;
    int rc = ex_prepare(d, &j);
    if (rc) return rc;
    for (size_t batch = 0; batch < d->batch_count; ++batch) ex_cols(&j, batch, 0, d->n);
    return OR_OK;
}

int or_gemm_ex_mt(const or_ex_desc *d, int threads) {
    ex_job j;
    int rc = ex_prepare(d, &j);
    if (rc) return rc;
    run_ranges(ex_range, &j, d->batch_count, d->n, threads);
    return OR_OK;
}

int or_gemm_ex_entries(const or_ex_desc *d, size_t count, const int64_t *batch, const int64_t *row,
                       const int64_t *col, uint8_t *out) {
    ex_job j;
    int rc = ex_prepare(d, &j);
    if (rc) return rc;
    for (size_t i = 0; i < count; ++i) {
        if (batch[i] < 0 || row[i] < 0 || col[i] < 0 || (size_t)batch[i] >= d->batch_count ||
            (size_t)row[i] >= d->m || (size_t)col[i] >= d->n)
            return OR_ERR_INVALID_ARGUMENT;
        or_scalar sum = ex_sum(&j, (size_t)batch[i], (size_t)row[i], (size_t)col[i]);
        size_t ci = (size_t)batch[i] * j.sc + lidx(j.cl, (size_t)row[i], (size_t)col[i]);
        or_scalar v = ex_final(d, sum, d->c, ci);
        or_write_scalar(out, d->c_type, i, &v);
    }
    return OR_OK;
}

/* gemmBatchedEx (src/gemm.zig:636-663): one gemmExCuda per pointer triple. */
int or_gemm_batched_ex(const or_ptr_batched_desc *p) {
    if (p->a_count != p->b_count || p->a_count != p->c_count) return OR_ERR_INVALID_BATCH_COUNT;
    for (size_t i = 0; i < p->a_count; ++i) {
        or_ex_desc one;
        memset(&one, 0, sizeof one);
        one.op_a = p->op_a; one.op_b = p->op_b; one.m = p->m; one.n = p->n; one.k = p->k;
        one.alpha = p->alpha;
        one.a = p->a[i]; one.a_len = p->a_lens[i]; one.a_type = p->a_type; one.lda = p->lda;
        one.b = p->b[i]; one.b_len = p->b_lens[i]; one.b_type = p->b_type; one.ldb = p->ldb;
        one.beta = p->beta;
        one.c = p->c[i]; one.c_len = p->c_lens[i]; one.c_type = p->c_type; one.ldc = p->ldc;
        one.compute_type = p->compute_type; one.layout = p->layout; one.algo = p->algo;
        one.batch_count = 1;
        int rc = or_gemm_ex(&one);
        if (rc) return rc;
    }
    return OR_OK;
}
