// capi.cu -- the C ABI of libgemm_sm100 (include/gemm_sm100.h).
//
// Mirrors the cuBLAS calls slang-gemm makes through src/cublas.zig
// (Context :78-90, sgemm :171-173, sgemmStridedBatched :195-197,
// gemmEx :227-229, gemmStridedBatchedEx :235-237, gemmBatchedEx :239-241)
// with cuBLAS argument checking and status codes, and routes each call to a
// B200 kernel: tcgen05 for f16/bf16/s8, FFMA for f32, a CUDA-core kernel for
// operands TMA cannot address, and a scale kernel for k == 0. There is no CPU
// compute path: without a usable sm_100 device every call fails.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "gs_internal.h"

namespace gs {

size_t in_elem_size(InKind k) { return k == IN_I8 ? 1 : ((k == IN_F32 || k == IN_TF32) ? 4 : 2); }
size_t out_elem_size(OutKind k) { return (k == OUT_F16 || k == OUT_BF16) ? 2 : 4; }

// ---- tensor-map encoder (driver entry point, resolved once) --------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encoder() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

bool encode_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t dim0, uint64_t dim1,
                    uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                    std::string *why, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn enc = get_encoder();
    if (!enc) {
        if (why) *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    cuuint64_t dims[3] = {dim0, dim1, dim2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        if (why) *why = "cuTensorMapEncodeTiled returned " + std::to_string(static_cast<int>(r));
        return false;
    }
    return true;
}

// ---- planning: validation and kernel choice (host only) -----------------

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

gs_status plan_gemm(const GemmDesc &d, Plan *plan, std::string *why) {
    plan->kernel = 0;
    if (d.m == 0 || d.n == 0 || d.batch == 0) return GS_STATUS_SUCCESS;
    if (d.k == 0) {
        plan->kernel = GS_KERNEL_SCALE;
        return GS_STATUS_SUCCESS;
    }
    if (d.in_kind == IN_F32) {
        plan->kernel = d.fast_tf32 && tf32_worthwhile(d) ? GS_KERNEL_TC_TF32 : GS_KERNEL_FFMA;
        return GS_STATUS_SUCCESS;
    }
    const long long es = static_cast<long long>(in_elem_size(d.in_kind));
    bool tma = true;
    if (!aligned16(d.A) || !aligned16(d.B)) tma = false;
    if ((d.lda * es) % 16 != 0 || (d.ldb * es) % 16 != 0) tma = false;
    if (d.batch > 1 && ((d.stride_a * es) % 16 != 0 || (d.stride_b * es) % 16 != 0)) tma = false;
    if (d.batch > 1 && (d.stride_a < 0 || d.stride_b < 0)) tma = false;
    plan->kernel = tma ? (d.in_kind == IN_F16 ? GS_KERNEL_TC_F16 : d.in_kind == IN_BF16 ? GS_KERNEL_TC_BF16 : GS_KERNEL_TC_I8)
                       : GS_KERNEL_SIMT;
    if (!tma && why) *why = "operands not 16-byte aligned for TMA; CUDA-core kernel";
    return GS_STATUS_SUCCESS;
}

}  // namespace gs

using namespace gs;


static gs_status fail(gs_handle h, gs_status st, const std::string &msg) {
    if (h) h->ctx.last_error = msg;
    return st;
}

static gs_status from_cuda(gs_handle h, cudaError_t e, const char *where) {
    if (e == cudaSuccess) return GS_STATUS_SUCCESS;
    std::string msg = std::string(where) + ": " + cudaGetErrorString(e);
    // a launcher that refused to grow a buffer under stream capture said why
    if (e == cudaErrorStreamCaptureUnsupported && h && !h->ctx.last_error.empty()) msg += " (" + h->ctx.last_error + ")";
    return fail(h, GS_STATUS_EXECUTION_FAILED, msg);
}

extern "C" {

const char *gs_status_name(gs_status s) {
    switch (s) {
    case GS_STATUS_SUCCESS: return "GS_STATUS_SUCCESS";
    case GS_STATUS_NOT_INITIALIZED: return "GS_STATUS_NOT_INITIALIZED";
    case GS_STATUS_ALLOC_FAILED: return "GS_STATUS_ALLOC_FAILED";
    case GS_STATUS_INVALID_VALUE: return "GS_STATUS_INVALID_VALUE";
    case GS_STATUS_ARCH_MISMATCH: return "GS_STATUS_ARCH_MISMATCH";
    case GS_STATUS_EXECUTION_FAILED: return "GS_STATUS_EXECUTION_FAILED";
    case GS_STATUS_INTERNAL_ERROR: return "GS_STATUS_INTERNAL_ERROR";
    case GS_STATUS_NOT_SUPPORTED: return "GS_STATUS_NOT_SUPPORTED";
    }
    return "GS_STATUS_UNKNOWN";
}

gs_status gs_select_device(const char *name_substr, int *device) {
    if (!device) return GS_STATUS_INVALID_VALUE;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    const bool any = name_substr == nullptr || name_substr[0] == '\0';
    bool matched = false;
    for (int d = 0; d < count; ++d) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, d) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (!any && std::strstr(prop.name, name_substr) == nullptr) continue;
        matched = true;
        if (prop.major != 10 || prop.minor != 0) continue;  // a later match may still be an sm_100 device
        if (cudaSetDevice(d) != cudaSuccess) {
            cudaGetLastError();
            return GS_STATUS_NOT_INITIALIZED;
        }
        *device = d;
        return GS_STATUS_SUCCESS;
    }
    return matched ? GS_STATUS_ARCH_MISMATCH : GS_STATUS_INVALID_VALUE;
}

gs_status gs_create(gs_handle *handle) {
    if (!handle) return GS_STATUS_INVALID_VALUE;
    *handle = nullptr;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    if (prop.major != 10 || prop.minor != 0) return GS_STATUS_ARCH_MISMATCH;
    gs_context *h = new (std::nothrow) gs_context();
    if (!h) return GS_STATUS_ALLOC_FAILED;
    h->ctx.device = dev;
    h->ctx.sm_count = prop.multiProcessorCount;
    if (cudaMalloc(&h->ctx.dev_err, 256) != cudaSuccess) {
        cudaGetLastError();
        delete h;
        return GS_STATUS_ALLOC_FAILED;
    }
    if (cudaMemset(h->ctx.dev_err, 0, 256) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(h->ctx.dev_err);
        delete h;
        return GS_STATUS_ALLOC_FAILED;
    }
    *handle = h;
    return GS_STATUS_SUCCESS;
}

gs_status gs_destroy(gs_handle h) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(h->ctx.device);
    cudaDeviceSynchronize();
    if (h->ctx.dev_err) cudaFree(h->ctx.dev_err);
    if (h->ctx.stage) cudaFree(h->ctx.stage);
    if (h->ctx.tmap_buf) cudaFree(h->ctx.tmap_buf);
    if (h->ctx.sk_buf) cudaFree(h->ctx.sk_buf);
    if (h->ctx.sk_counts) cudaFree(h->ctx.sk_counts);
    if (h->ctx.splitk_buf) cudaFree(h->ctx.splitk_buf);
    for (void *p : h->ctx.retired) cudaFree(p);
    if (h->ctx.tf32_buf) cudaFree(h->ctx.tf32_buf);
    if (h->ctx.h2d) cudaStreamDestroy(h->ctx.h2d);
    if (h->ctx.d2h) cudaStreamDestroy(h->ctx.d2h);
    if (h->ctx.ev_start) cudaEventDestroy(h->ctx.ev_start);
    if (h->ctx.ev_a) cudaEventDestroy(h->ctx.ev_a);
    for (int i = 0; i < Context::kMaxChunks; ++i) {
        if (h->ctx.ev_in[i]) cudaEventDestroy(h->ctx.ev_in[i]);
        if (h->ctx.ev_out[i]) cudaEventDestroy(h->ctx.ev_out[i]);
    }
    if (prev >= 0) cudaSetDevice(prev);
    delete h;
    return GS_STATUS_SUCCESS;
}

gs_status gs_set_stream(gs_handle h, void *stream) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    h->ctx.stream = static_cast<cudaStream_t>(stream);
    return GS_STATUS_SUCCESS;
}

gs_status gs_get_stream(gs_handle h, void **stream) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    if (!stream) return GS_STATUS_INVALID_VALUE;
    *stream = h->ctx.stream;
    return GS_STATUS_SUCCESS;
}

const char *gs_last_error(gs_handle h) { return h ? h->ctx.last_error.c_str() : "null handle"; }
uint32_t gs_last_kernels(gs_handle h) { return h ? h->ctx.last_kernels : 0u; }
uint64_t gs_launch_count(gs_handle h) { return h ? h->ctx.launches : 0u; }

gs_status gs_plan_shards(long long units, int parts, long long align, long long *offsets) {
    if (units < 0 || parts < 1 || align < 1 || !offsets) return GS_STATUS_INVALID_VALUE;
    offsets[0] = 0;
    for (int g = 1; g < parts; ++g) {
        long long cut = static_cast<long long>((static_cast<__int128>(units) * g) / parts);
        cut = (cut / align) * align;
        if (cut < offsets[g - 1]) cut = offsets[g - 1];
        offsets[g] = cut;
    }
    offsets[parts] = units;
    return GS_STATUS_SUCCESS;
}

gs_status gs_device_error(gs_handle h, uint32_t *word);

}  // extern "C"

// ---- argument decoding shared by the typed entry points ----------------

namespace gs {

// Maps (Atype, Btype, Ctype, computeType) onto a kernel family, or
// GS_STATUS_NOT_SUPPORTED (cf. the cuBLAS-supported set the reference bench
// enumerates, src/manifest.zig:404-410).
gs_status decode_types(int at, int bt, int ct, int comp, TypedArgs *t) {
    if (at != bt) return GS_STATUS_NOT_SUPPORTED;
    const bool c32f = comp == GS_COMPUTE_32F || comp == GS_COMPUTE_32F_PEDANTIC;
    if (at == GS_R_16F) {
        if ((c32f || comp == GS_COMPUTE_32F_FAST_16F) && ct == GS_R_32F) { *t = {IN_F16, OUT_F32}; return GS_STATUS_SUCCESS; }
        if ((c32f || comp == GS_COMPUTE_32F_FAST_16F) && ct == GS_R_16F) { *t = {IN_F16, OUT_F16}; return GS_STATUS_SUCCESS; }
        if ((comp == GS_COMPUTE_16F || comp == GS_COMPUTE_16F_PEDANTIC) && ct == GS_R_16F) { *t = {IN_F16, OUT_F16}; return GS_STATUS_SUCCESS; }
        return GS_STATUS_NOT_SUPPORTED;
    }
    if (at == GS_R_16BF) {
        if ((c32f || comp == GS_COMPUTE_32F_FAST_16BF) && ct == GS_R_32F) { *t = {IN_BF16, OUT_F32}; return GS_STATUS_SUCCESS; }
        if ((c32f || comp == GS_COMPUTE_32F_FAST_16BF) && ct == GS_R_16BF) { *t = {IN_BF16, OUT_BF16}; return GS_STATUS_SUCCESS; }
        return GS_STATUS_NOT_SUPPORTED;
    }
    if (at == GS_R_8I) {
        if ((comp == GS_COMPUTE_32I || comp == GS_COMPUTE_32I_PEDANTIC) && ct == GS_R_32I) { *t = {IN_I8, OUT_I32}; return GS_STATUS_SUCCESS; }
        return GS_STATUS_NOT_SUPPORTED;
    }
    if (at == GS_R_32F) {
        // FAST_TF32 permits TF32 products: large problems run on the tensor cores with three
        // tf32 products per f32 product (within the f32 tolerance), small ones on FFMA.
        if ((c32f || comp == GS_COMPUTE_32F_FAST_TF32) && ct == GS_R_32F) { *t = {IN_F32, OUT_F32}; return GS_STATUS_SUCCESS; }
        return GS_STATUS_NOT_SUPPORTED;
    }
    return GS_STATUS_NOT_SUPPORTED;
}

float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        float mag = static_cast<float>(m) * (1.0f / 16777216.0f);
        return sign ? -mag : mag;
    }
    if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e - 15u + 127u) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Reads alpha/beta from host memory according to the compute type.
void read_scalars(int comp, const void *alpha, const void *beta, Epilogue *ep) {
    std::memset(ep, 0, sizeof(*ep));
    if (comp == GS_COMPUTE_32I || comp == GS_COMPUTE_32I_PEDANTIC) {
        ep->alpha_i = *static_cast<const int32_t *>(alpha);
        ep->beta_i = *static_cast<const int32_t *>(beta);
        ep->beta_zero = ep->beta_i == 0;
        ep->identity = ep->alpha_i == 1 && ep->beta_zero;
        return;
    }
    if (comp == GS_COMPUTE_16F || comp == GS_COMPUTE_16F_PEDANTIC) {
        ep->alpha_f = half_bits_to_float(*static_cast<const uint16_t *>(alpha));
        ep->beta_f = half_bits_to_float(*static_cast<const uint16_t *>(beta));
    } else {
        ep->alpha_f = *static_cast<const float *>(alpha);
        ep->beta_f = *static_cast<const float *>(beta);
    }
    ep->beta_zero = ep->beta_f == 0.0f;
    ep->identity = ep->alpha_f == 1.0f && ep->beta_zero;
}

bool valid_op(int op) { return op == GS_OP_N || op == GS_OP_T || op == GS_OP_C; }

// Common cuBLAS argument checks (no handle, no device); fills the
// descriptor's shape fields.
gs_status check_shape_core(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int batch,
                           GemmDesc *d, std::string *why) {
    if (!valid_op(transa) || !valid_op(transb)) { *why = "invalid op"; return GS_STATUS_INVALID_VALUE; }
    if (m < 0 || n < 0 || k < 0 || batch < 0) { *why = "negative dimension"; return GS_STATUS_INVALID_VALUE; }
    const int a_rows = transa == GS_OP_N ? m : k;
    const int b_rows = transb == GS_OP_N ? k : n;
    if (lda < (a_rows > 1 ? a_rows : 1)) { *why = "lda too small"; return GS_STATUS_INVALID_VALUE; }
    if (ldb < (b_rows > 1 ? b_rows : 1)) { *why = "ldb too small"; return GS_STATUS_INVALID_VALUE; }
    if (ldc < (m > 1 ? m : 1)) { *why = "ldc too small"; return GS_STATUS_INVALID_VALUE; }
    // Row, column and K coordinates inside the kernels are 32-bit and run up
    // to one tile past the last row, column or K step.
    constexpr int kMaxDim = 0x7fffffff - 1024;
    if (m > 0 && n > 0 && batch > 0 && (m > kMaxDim || n > kMaxDim || k > kMaxDim)) {
        *why = "m, n and k are limited to 2^31 - 1025 (32-bit tile coordinates)";
        return GS_STATUS_NOT_SUPPORTED;
    }
    d->trans_a = transa == GS_OP_N ? 0 : 1;
    d->trans_b = transb == GS_OP_N ? 0 : 1;
    d->m = m;
    d->n = n;
    d->k = k;
    d->batch = batch;
    d->lda = lda;
    d->ldb = ldb;
    d->ldc = ldc;
    return GS_STATUS_SUCCESS;
}

gs_status check_shape(gs_handle h, int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int batch,
                      GemmDesc *d) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    std::string why;
    gs_status st = check_shape_core(transa, transb, m, n, k, lda, ldb, ldc, batch, d, &why);
    if (st != GS_STATUS_SUCCESS) return fail(h, st, why);
    return GS_STATUS_SUCCESS;
}

// Runs a validated strided (or single) GEMM.
gs_status run(gs_handle h, GemmDesc &d) {
    Context &ctx = h->ctx;
    ctx.last_kernels = 0;
    ctx.last_error.clear();
    Plan plan;
    std::string why;
    gs_status st = plan_gemm(d, &plan, &why);
    if (st != GS_STATUS_SUCCESS) return fail(h, st, why);
    cudaError_t e = cudaSuccess;
    switch (plan.kernel) {
    case 0: return GS_STATUS_SUCCESS;
    case GS_KERNEL_SCALE: e = launch_scale(ctx, d, nullptr); break;
    case GS_KERNEL_FFMA: e = launch_ffma(ctx, d); break;
    case GS_KERNEL_TC_TF32:
        e = launch_tf32(ctx, d);
        if (e == cudaErrorMemoryAllocation || e == cudaErrorInvalidValue) {
            // No room for the split operands, or a geometry TMA refuses: the exact FFMA kernel.
            cudaGetLastError();
            plan.kernel = GS_KERNEL_FFMA;
            e = launch_ffma(ctx, d);
        }
        break;
    case GS_KERNEL_SIMT: e = launch_simt(ctx, d, nullptr, nullptr, nullptr); break;
    default:
        e = launch_tc(ctx, d);
        if (e == cudaErrorInvalidValue && !ctx.last_error.empty()) {
            // Tensor-map encoding refused the geometry: use the CUDA-core kernel.
            cudaGetLastError();
            plan.kernel = GS_KERNEL_SIMT;
            e = launch_simt(ctx, d, nullptr, nullptr, nullptr);
        }
        break;
    }
    ctx.last_kernels |= plan.kernel;
    return from_cuda(h, e, "kernel launch");
}

}  // namespace gs

extern "C" {

gs_status gs_set_wait_limit(gs_handle h, long long cycles) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    h->ctx.spin_limit = cycles > 0 ? cycles : gs::kDefaultWaitLimitCycles;
    return GS_STATUS_SUCCESS;
}

gs_status gs_debug_skip_kblock(gs_handle h, int kblock) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    if (kblock < -1) return GS_STATUS_INVALID_VALUE;
    h->ctx.debug_skip_kb = kblock;
    return GS_STATUS_SUCCESS;
}

gs_status gs_device_error(gs_handle h, uint32_t *word) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    if (!word) return GS_STATUS_INVALID_VALUE;
    cudaError_t e = cudaStreamSynchronize(h->ctx.stream);
    if (e != cudaSuccess) return from_cuda(h, e, "stream synchronize");
    e = cudaMemcpy(word, h->ctx.dev_err, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    return from_cuda(h, e, "read device error word");
}

gs_status gs_gemm_strided_batched_ex(gs_handle h, int transa, int transb, int m, int n, int k, const void *alpha,
                                     const void *A, int Atype, int lda, long long strideA, const void *B, int Btype,
                                     int ldb, long long strideB, const void *beta, void *C, int Ctype, int ldc,
                                     long long strideC, int batchCount, int computeType, int algo) {
    // algo never changes results (src/gemm.zig:687 ignores it); it is used
    // only as a tile-shape hint for the tensor-core kernel.
    GemmDesc d{};
    d.algo = algo;
    gs_status st = check_shape(h, transa, transb, m, n, k, lda, ldb, ldc, batchCount, &d);
    if (st != GS_STATUS_SUCCESS) return st;
    TypedArgs t;
    st = decode_types(Atype, Btype, Ctype, computeType, &t);
    if (st != GS_STATUS_SUCCESS) return fail(h, st, "unsupported type / compute combination");
    if (t.in == IN_I8 && k > 131071) return fail(h, GS_STATUS_NOT_SUPPORTED, "INT8 with k > 131071 could overflow s32");
    if (!alpha || !beta) return fail(h, GS_STATUS_INVALID_VALUE, "alpha/beta must be host pointers");
    if (m == 0 || n == 0 || batchCount == 0) {
        h->ctx.last_kernels = 0;
        return GS_STATUS_SUCCESS;
    }
    if (!C || (k > 0 && (!A || !B))) return fail(h, GS_STATUS_INVALID_VALUE, "null matrix pointer");
    d.in_kind = t.in;
    d.out_kind = t.out;
    d.A = A;
    d.B = B;
    d.C = C;
    d.stride_a = strideA;
    d.stride_b = strideB;
    d.stride_c = strideC;
    d.fast_tf32 = t.in == IN_F32 && computeType == GS_COMPUTE_32F_FAST_TF32;
    read_scalars(computeType, alpha, beta, &d.ep);
    return run(h, d);
}

gs_status gs_plan_gemm_strided_batched_ex(int transa, int transb, int m, int n, int k, const void *A, int Atype,
                                          int lda, long long strideA, const void *B, int Btype, int ldb,
                                          long long strideB, const void *C, int Ctype, int ldc, long long strideC,
                                          int batchCount, int computeType, uint32_t *kernel) {
    if (!kernel) return GS_STATUS_INVALID_VALUE;
    *kernel = 0;
    GemmDesc d{};
    std::string why;
    gs_status st = check_shape_core(transa, transb, m, n, k, lda, ldb, ldc, batchCount, &d, &why);
    if (st != GS_STATUS_SUCCESS) return st;
    TypedArgs t;
    st = decode_types(Atype, Btype, Ctype, computeType, &t);
    if (st != GS_STATUS_SUCCESS) return st;
    if (t.in == IN_I8 && k > 131071) return GS_STATUS_NOT_SUPPORTED;
    if (m == 0 || n == 0 || batchCount == 0) return GS_STATUS_SUCCESS;
    if (!C || (k > 0 && (!A || !B))) return GS_STATUS_INVALID_VALUE;
    d.in_kind = t.in;
    d.out_kind = t.out;
    d.A = A;
    d.B = B;
    d.C = const_cast<void *>(C);
    d.fast_tf32 = t.in == IN_F32 && computeType == GS_COMPUTE_32F_FAST_TF32;
    d.stride_a = strideA;
    d.stride_b = strideB;
    d.stride_c = strideC;
    Plan plan;
    st = plan_gemm(d, &plan, &why);
    if (st == GS_STATUS_SUCCESS) *kernel = plan.kernel;
    return st;
}

gs_status gs_plan_tile(int transa, int transb, int m, int n, int k, int Atype, int Ctype, int computeType,
                       int batchCount, int algo, int sm_count, int *tile, int *k_slices) {
    if (!tile || !k_slices || sm_count < 2) return GS_STATUS_INVALID_VALUE;
    *tile = 0;
    *k_slices = 1;
    // tight leading dimensions of the stored operands (column-major)
    const int lda = std::max(1, transa ? k : m), ldb = std::max(1, transb ? n : k), ldc = std::max(1, m);
    GemmDesc d{};
    std::string why;
    gs_status st = check_shape_core(transa, transb, m, n, k, lda, ldb, ldc, batchCount, &d, &why);
    if (st != GS_STATUS_SUCCESS) return st;
    TypedArgs t;
    st = decode_types(Atype, Atype, Ctype, computeType, &t);
    if (st != GS_STATUS_SUCCESS) return st;
    if (t.in == IN_F32) return GS_STATUS_NOT_SUPPORTED;  // FFMA (or the FAST_TF32 split): not a tile of this kernel
    if (t.in == IN_I8 && k > 131071) return GS_STATUS_NOT_SUPPORTED;
    if (m == 0 || n == 0 || k == 0 || batchCount == 0) return GS_STATUS_SUCCESS;
    d.in_kind = t.in;
    d.out_kind = t.out;
    d.algo = algo;
    plan_tc_tile(d, sm_count, tile, k_slices);
    return GS_STATUS_SUCCESS;
}

gs_status gs_gemm_ex(gs_handle h, int transa, int transb, int m, int n, int k, const void *alpha, const void *A,
                     int Atype, int lda, const void *B, int Btype, int ldb, const void *beta, void *C, int Ctype, int ldc,
                     int computeType, int algo) {
    return gs_gemm_strided_batched_ex(h, transa, transb, m, n, k, alpha, A, Atype, lda, 0, B, Btype, ldb, 0, beta, C,
                                      Ctype, ldc, 0, 1, computeType, algo);
}

gs_status gs_sgemm(gs_handle h, int transa, int transb, int m, int n, int k, const float *alpha, const float *A,
                   int lda, const float *B, int ldb, const float *beta, float *C, int ldc) {
    return gs_gemm_strided_batched_ex(h, transa, transb, m, n, k, alpha, A, GS_R_32F, lda, 0, B, GS_R_32F, ldb, 0,
                                      beta, C, GS_R_32F, ldc, 0, 1, GS_COMPUTE_32F, GS_GEMM_DEFAULT);
}

gs_status gs_sgemm_strided_batched(gs_handle h, int transa, int transb, int m, int n, int k, const float *alpha,
                                   const float *A, int lda, long long strideA, const float *B, int ldb,
                                   long long strideB, const float *beta, float *C, int ldc, long long strideC,
                                   int batchCount) {
    return gs_gemm_strided_batched_ex(h, transa, transb, m, n, k, alpha, A, GS_R_32F, lda, strideA, B, GS_R_32F, ldb,
                                      strideB, beta, C, GS_R_32F, ldc, strideC, batchCount, GS_COMPUTE_32F,
                                      GS_GEMM_DEFAULT);
}

gs_status gs_hgemm(gs_handle h, int transa, int transb, int m, int n, int k, const uint16_t *alpha, const uint16_t *A,
                   int lda, const uint16_t *B, int ldb, const uint16_t *beta, uint16_t *C, int ldc) {
    return gs_gemm_strided_batched_ex(h, transa, transb, m, n, k, alpha, A, GS_R_16F, lda, 0, B, GS_R_16F, ldb, 0,
                                      beta, C, GS_R_16F, ldc, 0, 1, GS_COMPUTE_16F, GS_GEMM_DEFAULT);
}

gs_status gs_gemm_batched_ex(gs_handle h, int transa, int transb, int m, int n, int k, const void *alpha,
                             const void *const Aarray[], int Atype, int lda, const void *const Barray[], int Btype,
                             int ldb, const void *beta, void *const Carray[], int Ctype, int ldc, int batchCount,
                             int computeType, int algo) {
    GemmDesc d{};
    d.algo = algo;
    gs_status st = check_shape(h, transa, transb, m, n, k, lda, ldb, ldc, batchCount, &d);
    if (st != GS_STATUS_SUCCESS) return st;
    TypedArgs t;
    st = decode_types(Atype, Btype, Ctype, computeType, &t);
    if (st != GS_STATUS_SUCCESS) return fail(h, st, "unsupported type / compute combination");
    if (t.in == IN_I8 && k > 131071) return fail(h, GS_STATUS_NOT_SUPPORTED, "INT8 with k > 131071 could overflow s32");
    if (!alpha || !beta) return fail(h, GS_STATUS_INVALID_VALUE, "alpha/beta must be host pointers");
    Context &ctx = h->ctx;
    ctx.last_kernels = 0;
    if (m == 0 || n == 0 || batchCount == 0) return GS_STATUS_SUCCESS;
    if (!Carray || (k > 0 && (!Aarray || !Barray))) return fail(h, GS_STATUS_INVALID_VALUE, "null pointer array");
    d.in_kind = t.in;
    d.out_kind = t.out;
    read_scalars(computeType, alpha, beta, &d.ep);
    cudaError_t e;
    if (k == 0) {
        e = launch_scale(ctx, d, Carray);
        ctx.last_kernels |= GS_KERNEL_SCALE;
        return from_cuda(h, e, "kernel launch");
    }
    const long long es = static_cast<long long>(in_elem_size(t.in));
    const bool tc_types = t.in != IN_F32;
    const bool ld_ok = (d.lda * es) % 16 == 0 && (d.ldb * es) % 16 == 0;
    if (tc_types && ld_ok) {
        e = launch_tc_ptr_array(ctx, d, Aarray, Barray, Carray);
        ctx.last_kernels |= (t.in == IN_F16 ? GS_KERNEL_TC_F16 : t.in == IN_BF16 ? GS_KERNEL_TC_BF16 : GS_KERNEL_TC_I8);
    } else if (t.in == IN_F32) {
        e = launch_ffma_ptr(ctx, d, Aarray, Barray, Carray);
        ctx.last_kernels |= GS_KERNEL_FFMA;
    } else {
        e = launch_simt(ctx, d, Aarray, Barray, Carray);
        ctx.last_kernels |= GS_KERNEL_SIMT;
    }
    return from_cuda(h, e, "kernel launch");
}

}  // extern "C"
