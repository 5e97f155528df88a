/*
 * gemm_sm100.h -- C ABI of libgemm_sm100, a B200 (sm_100a) GEMM backend that
 * sits behind slang-gemm's cuBLAS-shaped API.
 *
 * Conventions (identical to cuBLAS and to slang-gemm's src/cublas.zig):
 *  - Matrices are column-major. Element (r, c) of a matrix with leading
 *    dimension ld lives at base[r + c*ld].
 *  - op values: GS_OP_N = 0, GS_OP_T = 1, GS_OP_C = 2 (src/cublas.zig:14-18).
 *    For real types GS_OP_C is identical to GS_OP_T.
 *  - Data / compute / algo enums carry CUDA's integer values
 *    (src/gemm.zig:14-113, pinned by tests/gemm_classic_extended.zig:6-16).
 *  - alpha and beta are HOST pointers whose type follows compute_type:
 *    float for GS_COMPUTE_32F*, int32_t for GS_COMPUTE_32I*, a uint16_t holding
 *    f16 bits for GS_COMPUTE_16F.
 *  - A, B, C (and the batched pointer arrays) are DEVICE pointers owned by the
 *    caller. All calls are asynchronous and ordered on the handle's stream.
 *  - beta == 0 means C is not read (cuBLAS semantics).
 *  - In strided-batched calls a stride of 0 re-uses the same matrix for every
 *    batch entry (cuBLAS semantics). The host-buffer mirror gs_host_gemm_ex
 *    instead follows src/gemm.zig, where 0 means "one matrix extent".
 *  - A handle is not thread-safe; use one handle per host thread.
 *
 * Return codes are cuBLAS's status values (cublasStatus_t).
 */
#ifndef GEMM_SM100_H
#define GEMM_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GS_VERSION_MAJOR 0
#define GS_VERSION_MINOR 1

typedef enum gs_status {
    GS_STATUS_SUCCESS = 0,
    GS_STATUS_NOT_INITIALIZED = 1,
    GS_STATUS_ALLOC_FAILED = 3,
    GS_STATUS_INVALID_VALUE = 7,
    GS_STATUS_ARCH_MISMATCH = 8,
    GS_STATUS_EXECUTION_FAILED = 13,
    GS_STATUS_INTERNAL_ERROR = 14,
    GS_STATUS_NOT_SUPPORTED = 15
} gs_status;

enum { GS_OP_N = 0, GS_OP_T = 1, GS_OP_C = 2 };

/* cudaDataType values (src/gemm.zig:14-49); the ones this backend computes on. */
enum {
    GS_R_32F = 0, GS_R_64F = 1, GS_R_16F = 2, GS_R_8I = 3, GS_R_32I = 10, GS_R_16BF = 14
};

/* cublasComputeType_t values (src/gemm.zig:53-67). */
enum {
    GS_COMPUTE_16F = 64, GS_COMPUTE_16F_PEDANTIC = 65,
    GS_COMPUTE_32F = 68, GS_COMPUTE_32F_PEDANTIC = 69,
    GS_COMPUTE_32F_FAST_16F = 74, GS_COMPUTE_32F_FAST_16BF = 75, GS_COMPUTE_32F_FAST_TF32 = 77,
    GS_COMPUTE_64F = 70, GS_COMPUTE_64F_PEDANTIC = 71,
    GS_COMPUTE_32I = 72, GS_COMPUTE_32I_PEDANTIC = 73
};

/* cublasGemmAlgo_t: accepted and ignored, as src/gemm.zig:687 ignores it. */
enum { GS_GEMM_DEFAULT = -1, GS_GEMM_DEFAULT_TENSOR_OP = 99 };

/* Row/column-major selector of the host-buffer mirror (src/gemm.zig:3-6). */
enum { GS_LAYOUT_ROW_MAJOR = 0, GS_LAYOUT_COL_MAJOR = 1 };

typedef struct gs_context *gs_handle;

/* ---------------------------------------------------------------------- */
/* Handle management. Replaces cublas.Context (src/cublas.zig:78-90).      */
/* ---------------------------------------------------------------------- */

/* Makes current the first CUDA device whose name contains name_substr (any
 * device when it is NULL or empty) and stores its index in *device. Replaces
 * the device choice of src/vulkan_runner.zig:1273-1299 (selectPhysicalDevice,
 * first device whose name contains the --device-substr needle). Statuses:
 * GS_STATUS_NOT_INITIALIZED when there is no CUDA device at all (the reference's
 * error.NoVulkanDevice), GS_STATUS_INVALID_VALUE when no name matches
 * (error.NoMatchingDevice), GS_STATUS_ARCH_MISMATCH when the matching devices
 * are not compute capability 10.0. Host only: allocates nothing. */
gs_status gs_select_device(const char *name_substr, int *device);

/* Creates a handle bound to the current CUDA device and the default stream.
 * Returns GS_STATUS_ARCH_MISMATCH when the device is not compute capability 10.0. */
gs_status gs_create(gs_handle *handle);
gs_status gs_destroy(gs_handle handle);
/* stream is a cudaStream_t (NULL = legacy default stream). */
gs_status gs_set_stream(gs_handle handle, void *stream);
gs_status gs_get_stream(gs_handle handle, void **stream);
/* Static, NUL-terminated name of a status value. */
const char *gs_status_name(gs_status status);
/* Human-readable detail of the last non-success status returned on this handle. */
const char *gs_last_error(gs_handle handle);
/* Bit set of kernels the last call launched (GS_KERNEL_* below); for tests/benchmarks. */
uint32_t gs_last_kernels(gs_handle handle);
/* Total number of kernel launches issued through this handle. */
uint64_t gs_launch_count(gs_handle handle);
/* Synchronises the handle's stream and returns the device error word that the
 * kernels' bounded waits write (0 = no error; bit 0 = a pipeline wait timed
 * out, bits 8..15 = where). The word is sticky for the handle's lifetime. */
gs_status gs_device_error(gs_handle handle, uint32_t *word);
/* Limit, in SM clock cycles, of every bounded wait inside this handle's
 * tensor-core kernels (default 4e9, about 2 s at the B200's top clock; a value
 * <= 0 restores the default). A wait that runs out records bit 0 and its site
 * in the device error word and ends the kernel early, with its in-flight copies
 * and MMAs drained and its tensor memory freed, instead of hanging the GPU: the
 * bounded counterpart of the reference's fence wait with no time limit
 * (src/vulkan_runner.zig:2197). Affects calls issued afterwards. */
gs_status gs_set_wait_limit(gs_handle handle, long long cycles);
/* Test hook for that failure path: with kblock >= 0 the tensor-core kernel's
 * TMA producer leaves K block `kblock` of its first tile unfilled (no
 * expect_tx, no copy) and issues nothing after it, so the MMA issuer's wait for
 * that stage runs out after the wait limit with no load left in flight. The
 * call's C is then incomplete and gs_device_error reports the timeout. -1 (the
 * default) turns it off. No counterpart in the reference. */
gs_status gs_debug_skip_kblock(gs_handle handle, int kblock);

enum {
    GS_KERNEL_TC_F16 = 1u << 0,   /* tcgen05 kind::f16, f16 operands */
    GS_KERNEL_TC_BF16 = 1u << 1,  /* tcgen05 kind::f16, bf16 operands */
    GS_KERNEL_TC_I8 = 1u << 2,    /* tcgen05 kind::i8 */
    GS_KERNEL_FFMA = 1u << 3,     /* register-blocked FFMA sgemm */
    GS_KERNEL_SIMT = 1u << 4,     /* generic CUDA-core kernel for operands TMA cannot address */
    GS_KERNEL_SCALE = 1u << 5,    /* C = beta*C for k == 0 */
    GS_KERNEL_TMAP = 1u << 6,     /* device-side tensor-map builder (pointer-array batches above
                                     GS_PTR_MAPS_IN_KERNEL_MAX_BATCH entries) */
    GS_KERNEL_TC_TF32 = 1u << 7,  /* COMPUTE_32F_FAST_TF32: operand split + tcgen05 kind::tf32 */
    GS_KERNEL_REDUCE = 1u << 8    /* split-K: sum of the tensor-core kernel's per-slice partials, alpha/beta */
};

/* ---------------------------------------------------------------------- */
/* cuBLAS-shaped device entry points                                       */
/* ---------------------------------------------------------------------- */

/* FP32 SGEMM, FFMA path. Replaces cublas.sgemm (src/cublas.zig:171-173) behind
 * gemm.sgemm (src/gemm.zig:286-317). */
gs_status gs_sgemm(gs_handle handle, int transa, int transb, int m, int n, int k,
                   const float *alpha, const float *A, int lda, const float *B, int ldb,
                   const float *beta, float *C, int ldc);

/* Strided-batched SGEMM. Replaces cublas.sgemmStridedBatched
 * (src/cublas.zig:195-197) behind gemm.sgemmStridedBatched (src/gemm.zig:479-481). */
gs_status gs_sgemm_strided_batched(gs_handle handle, int transa, int transb, int m, int n, int k,
                                   const float *alpha, const float *A, int lda, long long strideA,
                                   const float *B, int ldb, long long strideB, const float *beta,
                                   float *C, int ldc, long long strideC, int batchCount);

/* FP16 in / FP16 out with FP32 accumulation and f16 alpha/beta (bits), as
 * gemm.hgemm (src/gemm.zig:438-477). tcgen05 path. */
gs_status gs_hgemm(gs_handle handle, int transa, int transb, int m, int n, int k,
                   const uint16_t *alpha, const uint16_t *A, int lda, const uint16_t *B, int ldb,
                   const uint16_t *beta, uint16_t *C, int ldc);

/* Typed GEMM. Replaces cublas.gemmEx (src/cublas.zig:227-229, RawGemmExDesc
 * :243-266) behind gemm.gemmEx (src/gemm.zig:546-576). Supported combinations:
 *   A,B = R_16F,  C = R_32F or R_16F,  compute 32F / 32F_FAST_16F / 32F_PEDANTIC   (tcgen05)
 *   A,B = R_16BF, C = R_32F or R_16BF, compute 32F / 32F_FAST_16BF / 32F_PEDANTIC  (tcgen05)
 *   A,B = R_16F,  C = R_16F,           compute 16F (alpha/beta f16 bits)           (tcgen05)
 *   A,B = R_8I,   C = R_32I,           compute 32I / 32I_PEDANTIC                  (tcgen05)
 *   A,B,C = R_32F,                     compute 32F / 32F_PEDANTIC                  (FFMA)
 *   A,B,C = R_32F,                     compute 32F_FAST_TF32: problems of at least a GFLOP on the
 *                                      tensor cores, each f32 product as three tf32 products
 *                                      (hi*hi + hi*lo + lo*hi), K accumulated in chunks added in
 *                                      f32, within the FP32 tolerance; smaller ones on FFMA
 * Anything else returns GS_STATUS_NOT_SUPPORTED. INT8 requires k <= 131071 so
 * that the s32 accumulator cannot overflow. For every type a non-empty problem
 * with m, n or k above 2^31 - 1025 returns GS_STATUS_NOT_SUPPORTED (the
 * kernels' tile coordinates are 32-bit). */
gs_status gs_gemm_ex(gs_handle handle, int transa, int transb, int m, int n, int k,
                     const void *alpha, const void *A, int Atype, int lda,
                     const void *B, int Btype, int ldb, const void *beta,
                     void *C, int Ctype, int ldc, int computeType, int algo);

/* Strided-batched typed GEMM. Replaces cublas.gemmStridedBatchedEx
 * (src/cublas.zig:235-237) behind gemm.gemmStridedBatchedEx (src/gemm.zig:632-634). */
gs_status gs_gemm_strided_batched_ex(gs_handle handle, int transa, int transb, int m, int n, int k,
                                     const void *alpha, const void *A, int Atype, int lda, long long strideA,
                                     const void *B, int Btype, int ldb, long long strideB,
                                     const void *beta, void *C, int Ctype, int ldc, long long strideC,
                                     int batchCount, int computeType, int algo);

/* Pointer-array batched typed GEMM; Aarray/Barray/Carray are DEVICE arrays of
 * device pointers, as with cuBLAS. Replaces cublas.gemmBatchedEx
 * (src/cublas.zig:239-241, RawGemmBatchedExDesc :268-288) behind
 * gemm.gemmBatchedEx (src/gemm.zig:636-663). Tensor-core calls of at most
 * GS_PTR_MAPS_IN_KERNEL_MAX_BATCH entries are one launch: each CTA of the GEMM
 * kernel writes the per-entry tensor maps it uses into its own slots of the
 * handle's map buffer (3 * SMs * batchCount maps). Larger batches launch a map
 * builder (GS_KERNEL_TMAP) first. */
#define GS_PTR_MAPS_IN_KERNEL_MAX_BATCH 64

gs_status gs_gemm_batched_ex(gs_handle handle, int transa, int transb, int m, int n, int k,
                             const void *alpha, const void *const Aarray[], int Atype, int lda,
                             const void *const Barray[], int Btype, int ldb, const void *beta,
                             void *const Carray[], int Ctype, int ldc, int batchCount,
                             int computeType, int algo);

/* Validates a strided-batched typed GEMM exactly as gs_gemm_strided_batched_ex
 * does (same status codes) and reports in *kernel the GS_KERNEL_* bit it would
 * launch (0 for a no-op). Pure host logic: touches no device and needs no
 * handle, so callers can query the dispatch decision up front. */
gs_status gs_plan_gemm_strided_batched_ex(int transa, int transb, int m, int n, int k, const void *A, int Atype,
                                          int lda, long long strideA, const void *B, int Btype, int ldb,
                                          long long strideB, const void *C, int Ctype, int ldc, long long strideC,
                                          int batchCount, int computeType, uint32_t *kernel);

/* The tensor-core tile and K split a strided-batched typed GEMM of this shape
 * would use on a device with sm_count SMs, assuming tight leading dimensions
 * and 16-byte aligned operands: *tile = 1 (1-SM 128x256), 2 (2-SM 256x256
 * pair) or 3 (2-SM 256x512 wide pair), or 0 for a no-op; *k_slices = the
 * number of K slices (1 = no split-K). FP32 types (FFMA or the FAST_TF32
 * split) return GS_STATUS_NOT_SUPPORTED. Pure host logic, for tests and
 * capacity planning. */
gs_status gs_plan_tile(int transa, int transb, int m, int n, int k, int Atype, int Ctype, int computeType,
                       int batchCount, int algo, int sm_count, int *tile, int *k_slices);

/* Largest batchCount gs_gemm_batched_ex_noalloc accepts. */
#define GS_NOALLOC_MAX_BATCH 256

/* Pointer-array batched typed GEMM that allocates no memory and needs no
 * handle. No counterpart in the reference: it exists for callers that cannot
 * allocate device memory -- a framework whose caching allocator owns the GPU's
 * memory, a service with a fixed, pre-planned memory budget, or a
 * latency-critical path that must not pay the device-wide synchronisation
 * cudaMalloc/cudaFree can imply. Same arguments, types, semantics and status
 * codes as gs_gemm_batched_ex, plus the stream (a cudaStream_t) to run on.
 * Its scratch (per-batch tensor maps and status words: 3 * GS_NOALLOC_MAX_BATCH
 * * 128 + 256 = 98,560 bytes) is a static device array in the library that
 * every GPU loading the library holds until the process exits. Limit: batchCount <= GS_NOALLOC_MAX_BATCH;
 * larger batches return GS_STATUS_INVALID_VALUE and launch nothing.
 * The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture. All calls share the array and each clears the
 * words that must start at zero, so calls that overlap on the GPU (other
 * streams or host threads) race: order them on one stream. The array's address
 * is resolved once per device, so do not use this entry point on a device
 * after cudaDeviceReset in the same process. */
gs_status gs_gemm_batched_ex_noalloc(void *stream, int transa, int transb, int m, int n, int k, const void *alpha,
                                     const void *const Aarray[], int Atype, int lda, const void *const Barray[],
                                     int Btype, int ldb, const void *beta, void *const Carray[], int Ctype, int ldc,
                                     int batchCount, int computeType);

/* Reads the device error word of the last gs_gemm_batched_ex_noalloc call on
 * the current device, after synchronising `stream` (the stream that call ran
 * on): 0 = no error; bit 0 = a pipeline wait in the kernel gave up, bits 8..15
 * = where (the word gs_device_error reads for a handle). The call returned
 * success before the kernel ran, so this is how such a caller learns that a
 * kernel ended early and C is incomplete. Valid until the next no-allocation
 * call on the device clears it. No counterpart in the reference; allocates
 * nothing. */
gs_status gs_noalloc_device_error(void *stream, uint32_t *word);

/* ---------------------------------------------------------------------- */
/* Host-buffer mirror of gemm.gemmEx                                       */
/* ---------------------------------------------------------------------- */

/* Mirrors ExDesc (src/gemm.zig:236-261): host byte buffers with their lengths,
 * row- or column-major layout, f64 complex alpha/beta (only .re is used by the
 * real types computed here) and src/gemm.zig's stride convention (0 = extent). */
typedef struct gs_ex_desc {
    int op_a, op_b;
    size_t m, n, k;
    double alpha_re, alpha_im;
    const void *a; size_t a_len; int a_type; size_t lda;
    const void *b; size_t b_len; int b_type; size_t ldb;
    double beta_re, beta_im;
    void *c; size_t c_len; int c_type; size_t ldc;
    int compute_type;
    int layout;
    size_t batch_count;
    size_t stride_a, stride_b, stride_c;
    int algo;
} gs_ex_desc;

/* Drop-in for gemm.gemmEx / gemm.gemmStridedBatchedEx over HOST buffers
 * (src/gemm.zig:546, :632): validates like validateByteSliceLen
 * (src/gemm.zig:769-775), copies A, B (and C when beta != 0) to the device,
 * runs the device path on the handle's stream, copies C back and synchronises.
 * Device staging buffers are owned and reused by the handle. */
gs_status gs_host_gemm_ex(gs_handle handle, const gs_ex_desc *desc);

/* Mirrors PointerBatchedExDesc (src/gemm.zig:263-284): per-entry HOST byte
 * buffers with their lengths; counts must agree (else InvalidBatchCount). */
typedef struct gs_ptr_batched_desc {
    int op_a, op_b;
    size_t m, n, k;
    double alpha_re, alpha_im;
    const void *const *a; const size_t *a_lens; size_t a_count; int a_type; size_t lda;
    const void *const *b; const size_t *b_lens; size_t b_count; int b_type; size_t ldb;
    double beta_re, beta_im;
    void *const *c; const size_t *c_lens; size_t c_count; int c_type; size_t ldc;
    int compute_type;
    int layout;
    int algo;
} gs_ptr_batched_desc;

/* Drop-in for gemm.gemmBatchedEx (src/gemm.zig:636-663) over host buffers:
 * the entries' A, B (and C when read) are packed into the handle's device
 * staging, computed by one strided-batched call and copied back. Like the
 * reference's entry-by-entry loop, when entry i fails validation the entries
 * before it are still computed and written back, and the call returns
 * GS_STATUS_INVALID_VALUE; entry i and later are untouched. Synchronous. */
gs_status gs_host_gemm_batched_ex(gs_handle handle, const gs_ptr_batched_desc *desc);

/* ---------------------------------------------------------------------- */
/* Multi-GPU sharding plan (pure host logic)                               */
/* ---------------------------------------------------------------------- */

/* Splits `units` (batch entries, or columns of B and C) over `parts` devices
 * as [floor(g*units/parts), floor((g+1)*units/parts)), rounding interior cut
 * points down to a multiple of `align` (1 = no rounding). Writes parts+1
 * offsets into `offsets`. Used by the batch split of strided / pointer-array
 * calls and by the column split of one large GEMM. */
gs_status gs_plan_shards(long long units, int parts, long long align, long long *offsets);

/* ---------------------------------------------------------------------- */
/* Single-process multi-GPU calls                                          */
/* ---------------------------------------------------------------------- */
/* No reference counterpart: slang-gemm drives one device
 * (src/vulkan_runner.zig:1273-1299). These split the calls above over several
 * GPUs of one box from ONE host thread, one stream per device, and return
 * when every device is done. Neither split needs a reduction:
 *  - batched calls: device devs[g] computes batch entries
 *    [off[g], off[g+1]) with off = gs_plan_shards(batchCount, ngpu, 1);
 *  - gs_gemm_ex_colsplit_multi: device devs[g] computes the column block
 *    C[:, off[g]:off[g+1]] with off = gs_plan_shards(n, ngpu, GS_COLSPLIT_ALIGN),
 *    reading all of A and the matching columns of op(B).
 * Every pointer in A[], B[], C[] (and the device pointer arrays of the
 * pointer-array call) is the base of the WHOLE problem's buffer on device
 * devs[g] -- the same leading dimensions and strides as the single-GPU call --
 * and that device reads and writes only its own shard, so a caller may fill
 * just the shard region. No kernel reads another GPU's memory.
 * gather_to: -1 leaves each block on its device; an index g into devs copies
 * every other device's block of C into C[g] (NCCL point-to-point, loaded at
 * run time); GS_GATHER_ALL does that for every device. Gathering needs a dense
 * C (ldc == m and, when batched, strideC == m*n); otherwise it returns
 * GS_STATUS_NOT_SUPPORTED before launching anything. alpha/beta are host
 * pointers as in the single-GPU calls. The caller's current device is
 * restored on return. */
#define GS_MULTI_MAX_GPUS 64
#define GS_GATHER_ALL (-2)
#define GS_COLSPLIT_ALIGN 256

typedef struct gs_multi *gs_multi_handle;

/* Creates one gs_handle and one non-blocking stream per device in devs[0..ngpu). */
gs_status gs_multi_create(gs_multi_handle *handle, int ngpu, const int *devs);
gs_status gs_multi_destroy(gs_multi_handle handle);
const char *gs_multi_last_error(gs_multi_handle handle);
/* Per-device times (ms, CUDA events on each device's stream) of the last call:
 * the GEMM alone and GEMM + gather. Either array may be NULL; each holds ngpu
 * entries, 0 for a device that had no shard. */
gs_status gs_multi_last_times(gs_multi_handle handle, float *gemm_ms, float *total_ms);

gs_status gs_gemm_strided_batched_ex_multi(gs_multi_handle handle, int transa, int transb, int m, int n, int k,
                                           const void *alpha, const void *const A[], int Atype, int lda,
                                           long long strideA, const void *const B[], int Btype, int ldb,
                                           long long strideB, const void *beta, void *const C[], int Ctype, int ldc,
                                           long long strideC, int batchCount, int computeType, int algo,
                                           int gather_to);

/* Aarray[g] etc. are device-devs[g] arrays of batchCount device pointers
 * (entries outside the device's shard are not read). No gather: the C
 * matrices of a pointer-array call need not form one buffer. */
gs_status gs_gemm_batched_ex_multi(gs_multi_handle handle, int transa, int transb, int m, int n, int k,
                                   const void *alpha, const void *const *const Aarray[], int Atype, int lda,
                                   const void *const *const Barray[], int Btype, int ldb, const void *beta,
                                   void *const *const Carray[], int Ctype, int ldc, int batchCount, int computeType,
                                   int algo);

gs_status gs_gemm_ex_colsplit_multi(gs_multi_handle handle, int transa, int transb, int m, int n, int k,
                                    const void *alpha, const void *const A[], int Atype, int lda,
                                    const void *const B[], int Btype, int ldb, const void *beta, void *const C[],
                                    int Ctype, int ldc, int computeType, int algo, int gather_to);

#ifdef __cplusplus
}
#endif
#endif /* GEMM_SM100_H */
