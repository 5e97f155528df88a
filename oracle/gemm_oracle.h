/*
 * gemm_oracle.h -- CPU restatement of slang-gemm's scalar GEMM reference
 * (src/gemm.zig), used ONLY as a test checker and as the timed CPU baseline.
 *
 * TEST INFRASTRUCTURE. Nothing in the product library links or calls this
 * code. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline
 * leg and its `--impl reference` arm) load liboracle_gemm.so.
 *
 * Parity status: the reference is Zig 0.16 + Bazel and cannot be built in this
 * image, so the restatement is pinned by the reference's own known-answer
 * tests (tests/gemm_correctness.zig:30-44, tests/gemm_classic_extended.zig:6-16,
 * :129-143) and by the cross-check restatements those tests carry
 * (tests/gemm_correctness.zig:243-286 `referenceReal`); see tests/golden/.
 *
 * Conventions follow src/gemm.zig exactly:
 *  - MatrixLayout {offset,row_stride,col_stride}: index = offset + r*rs + c*cs
 *    (src/gemm.zig:155-170).
 *  - stride 0 in a batched descriptor means "one matrix extent"
 *    (src/gemm.zig:524-526, :679-681).
 *  - gemm(f32) accumulates in f32 in sequential k order, then writes
 *    alpha*sum + beta*c in f32 (src/gemm.zig:523-544).
 *  - gemmEx decodes each element to an f64 complex Scalar, accumulates in
 *    f64 in sequential k order, forms alpha*sum + beta*old in f64 and rounds
 *    once into c_type (src/gemm.zig:671-706, :797-896).
 */
#ifndef GEMM_ORACLE_H
#define GEMM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Layout / Op enums (src/gemm.zig:3-12). */
enum { OR_ROW_MAJOR = 0, OR_COL_MAJOR = 1 };
enum { OR_OP_N = 0, OR_OP_T = 1, OR_OP_C = 2 };

/* DataType values equal CUDA's cudaDataType (src/gemm.zig:14-49). */
enum {
    OR_R_32F = 0, OR_R_64F = 1, OR_R_16F = 2, OR_R_8I = 3, OR_C_32F = 4,
    OR_C_64F = 5, OR_C_16F = 6, OR_C_8I = 7, OR_R_8U = 8, OR_C_8U = 9,
    OR_R_32I = 10, OR_C_32I = 11, OR_R_32U = 12, OR_C_32U = 13,
    OR_R_16BF = 14, OR_C_16BF = 15, OR_R_4I = 16, OR_C_4I = 17, OR_R_4U = 18,
    OR_C_4U = 19, OR_R_16I = 20, OR_C_16I = 21, OR_R_16U = 22, OR_C_16U = 23,
    OR_R_64I = 24, OR_C_64I = 25, OR_R_64U = 26, OR_C_64U = 27,
    OR_R_8F_E4M3 = 28, OR_R_8F_E5M2 = 29, OR_R_8F_UE8M0 = 30,
    OR_R_6F_E2M3 = 31, OR_R_6F_E3M2 = 32, OR_R_4F_E2M1 = 33
};

/* Error returns mirror the Zig error set used on this path. */
enum {
    OR_OK = 0,
    OR_ERR_INVALID_BATCH_COUNT = 1, /* error.InvalidBatchCount */
    OR_ERR_INVALID_STRIDE = 2,      /* error.InvalidStride */
    OR_ERR_BUFFER_TOO_SMALL = 3,    /* error.BufferTooSmall */
    OR_ERR_INVALID_TYPE = 4,        /* error.InvalidType */
    OR_ERR_INVALID_ARGUMENT = 5     /* bad entry index for the sampled checker */
};

typedef struct or_layout {
    size_t offset;
    size_t row_stride;
    size_t col_stride;
} or_layout;

typedef struct or_scalar {
    double re;
    double im;
} or_scalar;

/* ExDesc (src/gemm.zig:236-261); byte slices carry their lengths. */
typedef struct or_ex_desc {
    int op_a, op_b;
    size_t m, n, k;
    or_scalar alpha;
    const uint8_t *a; size_t a_len; int a_type; size_t lda;
    const uint8_t *b; size_t b_len; int b_type; size_t ldb;
    or_scalar beta;
    uint8_t *c; size_t c_len; int c_type; size_t ldc;
    int compute_type;              /* ignored, as in src/gemm.zig:686 */
    int layout;                    /* OR_ROW_MAJOR / OR_COL_MAJOR */
    size_t batch_count;
    size_t stride_a, stride_b, stride_c;
    int algo;                      /* ignored, as in src/gemm.zig:687 */
} or_ex_desc;

/* PointerBatchedExDesc (src/gemm.zig:263-284). */
typedef struct or_ptr_batched_desc {
    int op_a, op_b;
    size_t m, n, k;
    or_scalar alpha;
    const uint8_t *const *a; const size_t *a_lens; size_t a_count; int a_type; size_t lda;
    const uint8_t *const *b; const size_t *b_lens; size_t b_count; int b_type; size_t ldb;
    or_scalar beta;
    uint8_t *const *c; const size_t *c_lens; size_t c_count; int c_type; size_t ldc;
    int compute_type;
    int layout;
    int algo;
} or_ptr_batched_desc;

/* ---- layout helpers (src/gemm.zig:165-191, :708-711) ---- */
or_layout or_matrix_layout(int layout, size_t ld);
size_t or_stored_rows(int op, size_t rows, size_t cols);
size_t or_stored_cols(int op, size_t rows, size_t cols);
size_t or_minimum_ld(int layout, size_t rows, size_t cols);
size_t or_matrix_extent(or_layout l, size_t rows, size_t cols);
size_t or_element_size(int data_type);
int or_is_complex_type(int data_type);

/* ---- codecs (src/gemm.zig:797-1010) ---- */
uint16_t or_f32_to_f16_bits(float v);
float or_f16_bits_to_f32(uint16_t bits);
uint16_t or_f32_to_bf16_bits(float v);
float or_bf16_bits_to_f32(uint16_t bits);
float or_fp8_e4m3_to_f32(uint8_t bits);
float or_fp8_e5m2_to_f32(uint8_t bits);
void or_read_scalar(const uint8_t *data, int data_type, size_t index, or_scalar *out);
void or_write_scalar(uint8_t *data, int data_type, size_t index, const or_scalar *value);

/* ---- scalar GEMMs ---- */
/* gemm(f32) with explicit layouts, batching and strides (src/gemm.zig:523-544). */
int or_gemm_f32(int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                const float *a, size_t a_len, or_layout al,
                const float *b, size_t b_len, or_layout bl, float beta,
                float *c, size_t c_len, or_layout cl,
                size_t batch_count, size_t stride_a, size_t stride_b, size_t stride_c);
/* sgemm (src/gemm.zig:286-317) and sgemmStridedBatched (:479-481). */
int or_sgemm(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
             const float *a, size_t a_len, size_t lda, const float *b, size_t b_len, size_t ldb,
             float beta, float *c, size_t c_len, size_t ldc);
int or_sgemm_strided_batched(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                             const float *a, size_t a_len, size_t lda, size_t stride_a,
                             const float *b, size_t b_len, size_t ldb, size_t stride_b, float beta,
                             float *c, size_t c_len, size_t ldc, size_t stride_c, size_t batch_count);
/* Multithreaded sgemm: same per-element arithmetic as or_gemm_f32 (bit-identical),
 * columns split over `threads` POSIX threads. */
int or_sgemm_strided_batched_mt(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, float alpha,
                                const float *a, size_t a_len, size_t lda, size_t stride_a,
                                const float *b, size_t b_len, size_t ldb, size_t stride_b, float beta,
                                float *c, size_t c_len, size_t ldc, size_t stride_c, size_t batch_count,
                                int threads);
/* hgemm (src/gemm.zig:438-477): f16 bits in/out, f32 accumulation. */
int or_hgemm(int layout, int op_a, int op_b, size_t m, size_t n, size_t k, uint16_t alpha,
             const uint16_t *a, size_t lda, const uint16_t *b, size_t ldb, uint16_t beta,
             uint16_t *c, size_t ldc);
/* gemmExLegacy (src/gemm.zig:608-630): u16 inputs (f16 or bf16), f32 accumulation. */
int or_gemm_ex_legacy(int bf16_input, int op_a, int op_b, size_t m, size_t n, size_t k,
                      const uint16_t *a, size_t a_len, or_layout al,
                      const uint16_t *b, size_t b_len, or_layout bl,
                      float *c, size_t c_len, or_layout cl, float alpha, float beta,
                      size_t batch_count, size_t stride_a, size_t stride_b, size_t stride_c);
/* gemmEx / gemmStridedBatchedEx -> gemmExCuda (src/gemm.zig:546-606, :632-634, :671-706). */
int or_gemm_ex(const or_ex_desc *desc);
/* Same arithmetic, columns split over `threads` POSIX threads (bit-identical to or_gemm_ex). */
int or_gemm_ex_mt(const or_ex_desc *desc, int threads);
/* gemmBatchedEx (src/gemm.zig:636-663). */
int or_gemm_batched_ex(const or_ptr_batched_desc *desc);
/* Sampled checker: for each (batch,row,col) entry write into `out` (packed, c_type
 * encoded, one element per entry) exactly what gemmExCuda would store there, reading
 * the old C value from desc->c. desc->c is not modified. */
int or_gemm_ex_entries(const or_ex_desc *desc, size_t count, const int64_t *batch,
                       const int64_t *row, const int64_t *col, uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif /* GEMM_ORACLE_H */
