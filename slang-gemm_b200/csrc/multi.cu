// multi.cu -- single-process multi-GPU entry points (one host thread, one
// stream per device, synchronous on return).
//
// The reference drives exactly one device (src/vulkan_runner.zig:1273-1299);
// these calls are the sharding its GEMM contract allows because no partition
// needs a reduction:
//  - strided / pointer-array batches: device g computes batch entries
//    [floor(g*B/G), floor((g+1)*B/G)) of the same call
//    (gemm.gemmStridedBatchedEx / gemmBatchedEx, src/gemm.zig:632-663);
//  - one large GEMM: device g computes the column block C[:, j0:j1] from all
//    of A and B[:, j0:j1] (gemm.gemmEx, src/gemm.zig:546-576).
// Every operand pointer is the base of the WHOLE problem's buffer on that
// device; a device reads and writes only its shard, so a caller may fill only
// the shard region. NCCL (loaded at run time) moves C blocks point to point
// only when the caller asks for C on one device (gather_to >= 0) or on all
// (GS_GATHER_ALL). No kernel reads another GPU's memory.
#include <dlfcn.h>

#include <cstring>
#include <new>
#include <string>
#include <vector>

#include <nccl.h>

#include "gs_internal.h"

namespace {

// NCCL entry points resolved with dlopen, so that the library loads (and the
// single-GPU calls work) on a machine without NCCL.
struct NcclApi {
    bool tried = false, ok = false;
    std::string why;
    ncclResult_t (*comm_init_all)(ncclComm_t *, int, const int *) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

NcclApi &nccl() {
    static NcclApi api;
    if (api.tried) return api;
    api.tried = true;
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        api.why = "libnccl.so.2 not found";
        return api;
    }
    auto sym = [&](const char *name) { return dlsym(lib, name); };
    api.comm_init_all = reinterpret_cast<decltype(api.comm_init_all)>(sym("ncclCommInitAll"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.comm_init_all && api.comm_destroy && api.group_start && api.group_end && api.send && api.recv &&
             api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks a needed symbol";
    return api;
}

size_t elem_bytes(int t) {
    switch (t) {
    case GS_R_16F: case GS_R_16BF: return 2;
    case GS_R_32F: case GS_R_32I: return 4;
    case GS_R_8I: return 1;
    case GS_R_64F: return 8;
    default: return 0;
    }
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    DeviceGuard() { cudaGetDevice(&prev); }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

struct gs_multi {
    int ngpu = 0;
    std::vector<int> devs;
    std::vector<gs_handle> h;
    std::vector<cudaStream_t> stream;
    std::vector<cudaEvent_t> ev0, ev1, ev2;  // start, GEMM done, gather done
    std::vector<float> gemm_ms, total_ms;
    std::vector<ncclComm_t> comms;             // created on the first gather
    std::string last_error;
};

namespace {

gs_status fail(gs_multi *mh, gs_status st, const std::string &why) {
    mh->last_error = why;
    return st;
}

// Waits for every device's stream and collects per-device times and the
// handles' device error words.
gs_status finish(gs_multi *mh, const std::vector<int> &active, bool gathered) {
    gs_status st = GS_STATUS_SUCCESS;
    for (int g = 0; g < mh->ngpu; ++g) {
        cudaSetDevice(mh->devs[g]);
        cudaError_t e = cudaStreamSynchronize(mh->stream[g]);
        mh->gemm_ms[g] = mh->total_ms[g] = 0.0f;
        if (e != cudaSuccess) {
            mh->last_error = std::string("device ") + std::to_string(mh->devs[g]) + ": " + cudaGetErrorString(e);
            st = GS_STATUS_EXECUTION_FAILED;
            continue;
        }
        if (active[g]) {
            cudaEventElapsedTime(&mh->gemm_ms[g], mh->ev0[g], mh->ev1[g]);
            mh->total_ms[g] = mh->gemm_ms[g];
            if (gathered) cudaEventElapsedTime(&mh->total_ms[g], mh->ev0[g], mh->ev2[g]);
        }
        uint32_t word = 0;
        if (gs_device_error(mh->h[g], &word) == GS_STATUS_SUCCESS && word != 0) {
            mh->last_error = std::string("device ") + std::to_string(mh->devs[g]) + ": device error word " +
                             std::to_string(word);
            st = GS_STATUS_EXECUTION_FAILED;
        }
    }
    return st;
}

gs_status ensure_comms(gs_multi *mh) {
    if (!mh->comms.empty()) return GS_STATUS_SUCCESS;
    NcclApi &api = nccl();
    if (!api.ok) return fail(mh, GS_STATUS_NOT_SUPPORTED, "gather needs NCCL: " + api.why);
    std::vector<ncclComm_t> comms(mh->ngpu, nullptr);
    ncclResult_t r = api.comm_init_all(comms.data(), mh->ngpu, mh->devs.data());
    if (r != ncclSuccess) return fail(mh, GS_STATUS_EXECUTION_FAILED, std::string("ncclCommInitAll: ") + api.error_string(r));
    mh->comms = comms;
    return GS_STATUS_SUCCESS;
}

// Point-to-point gather of byte ranges: device g owns [off[g], off[g]+len[g])
// of C; every destination receives every other device's range in place.
gs_status gather_ranges(gs_multi *mh, void *const C[], const std::vector<size_t> &off, const std::vector<size_t> &len,
                        int gather_to) {
    gs_status st = ensure_comms(mh);
    if (st != GS_STATUS_SUCCESS) return st;
    NcclApi &api = nccl();
    ncclResult_t r = api.group_start();
    for (int g = 0; g < mh->ngpu && r == ncclSuccess; ++g) {
        if (!len[g]) continue;
        for (int d = 0; d < mh->ngpu && r == ncclSuccess; ++d) {
            if (d == g || (gather_to >= 0 && d != gather_to)) continue;
            r = api.send(static_cast<const char *>(C[g]) + off[g], len[g], ncclUint8, d, mh->comms[g], mh->stream[g]);
            if (r == ncclSuccess)
                r = api.recv(static_cast<char *>(C[d]) + off[g], len[g], ncclUint8, g, mh->comms[d], mh->stream[d]);
        }
    }
    ncclResult_t r2 = api.group_end();
    if (r == ncclSuccess) r = r2;
    if (r != ncclSuccess) return fail(mh, GS_STATUS_EXECUTION_FAILED, std::string("NCCL gather: ") + api.error_string(r));
    return GS_STATUS_SUCCESS;
}

gs_status check_common(gs_multi *mh, const void *A, const void *B, const void *C, int gather_to) {
    if (!mh) return GS_STATUS_NOT_INITIALIZED;
    if (!A || !B || !C) return fail(mh, GS_STATUS_INVALID_VALUE, "operand pointer arrays must not be NULL");
    if (gather_to < GS_GATHER_ALL || gather_to >= mh->ngpu)
        return fail(mh, GS_STATUS_INVALID_VALUE, "gather_to must be -1 (none), GS_GATHER_ALL or an index into devs");
    return GS_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

gs_status gs_multi_create(gs_multi_handle *out, int ngpu, const int *devs) {
    if (!out) return GS_STATUS_INVALID_VALUE;
    *out = nullptr;
    if (ngpu < 1 || ngpu > GS_MULTI_MAX_GPUS || !devs) return GS_STATUS_INVALID_VALUE;
    for (int i = 0; i < ngpu; ++i) {
        if (devs[i] < 0) return GS_STATUS_INVALID_VALUE;
        for (int j = 0; j < i; ++j)
            if (devs[i] == devs[j]) return GS_STATUS_INVALID_VALUE;
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    for (int i = 0; i < ngpu; ++i)
        if (devs[i] >= count) return GS_STATUS_INVALID_VALUE;
    gs_multi *mh = new (std::nothrow) gs_multi();
    if (!mh) return GS_STATUS_ALLOC_FAILED;
    mh->ngpu = ngpu;
    mh->devs.assign(devs, devs + ngpu);
    mh->h.assign(ngpu, nullptr);
    mh->stream.assign(ngpu, nullptr);
    mh->ev0.assign(ngpu, nullptr);
    mh->ev1.assign(ngpu, nullptr);
    mh->ev2.assign(ngpu, nullptr);
    mh->gemm_ms.assign(ngpu, 0.0f);
    mh->total_ms.assign(ngpu, 0.0f);
    DeviceGuard guard;
    gs_status st = GS_STATUS_SUCCESS;
    for (int g = 0; g < ngpu && st == GS_STATUS_SUCCESS; ++g) {
        if (cudaSetDevice(devs[g]) != cudaSuccess) {
            cudaGetLastError();
            st = GS_STATUS_NOT_INITIALIZED;
            break;
        }
        st = gs_create(&mh->h[g]);
        if (st != GS_STATUS_SUCCESS) break;
        if (cudaStreamCreateWithFlags(&mh->stream[g], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreate(&mh->ev0[g]) != cudaSuccess || cudaEventCreate(&mh->ev1[g]) != cudaSuccess ||
            cudaEventCreate(&mh->ev2[g]) != cudaSuccess) {
            cudaGetLastError();
            st = GS_STATUS_ALLOC_FAILED;
            break;
        }
        st = gs_set_stream(mh->h[g], mh->stream[g]);
    }
    if (st != GS_STATUS_SUCCESS) {
        gs_multi_destroy(mh);
        return st;
    }
    *out = mh;
    return GS_STATUS_SUCCESS;
}

gs_status gs_multi_destroy(gs_multi_handle mh) {
    if (!mh) return GS_STATUS_NOT_INITIALIZED;
    DeviceGuard guard;
    for (int g = 0; g < mh->ngpu; ++g) {
        cudaSetDevice(mh->devs[g]);
        if (mh->stream[g]) cudaStreamSynchronize(mh->stream[g]);
    }
    if (!mh->comms.empty()) {
        NcclApi &api = nccl();
        for (ncclComm_t c : mh->comms)
            if (c) api.comm_destroy(c);
    }
    for (int g = 0; g < mh->ngpu; ++g) {
        cudaSetDevice(mh->devs[g]);
        if (mh->h[g]) gs_destroy(mh->h[g]);
        if (mh->ev0[g]) cudaEventDestroy(mh->ev0[g]);
        if (mh->ev1[g]) cudaEventDestroy(mh->ev1[g]);
        if (mh->ev2[g]) cudaEventDestroy(mh->ev2[g]);
        if (mh->stream[g]) cudaStreamDestroy(mh->stream[g]);
    }
    delete mh;
    return GS_STATUS_SUCCESS;
}

const char *gs_multi_last_error(gs_multi_handle mh) { return mh ? mh->last_error.c_str() : "null handle"; }

gs_status gs_multi_last_times(gs_multi_handle mh, float *gemm_ms, float *total_ms) {
    if (!mh) return GS_STATUS_NOT_INITIALIZED;
    for (int g = 0; g < mh->ngpu; ++g) {
        if (gemm_ms) gemm_ms[g] = mh->gemm_ms[g];
        if (total_ms) total_ms[g] = mh->total_ms[g];
    }
    return GS_STATUS_SUCCESS;
}

gs_status gs_gemm_strided_batched_ex_multi(gs_multi_handle mh, int transa, int transb, int m, int n, int k,
                                           const void *alpha, const void *const A[], int Atype, int lda,
                                           long long strideA, const void *const B[], int Btype, int ldb,
                                           long long strideB, const void *beta, void *const C[], int Ctype, int ldc,
                                           long long strideC, int batchCount, int computeType, int algo,
                                           int gather_to) {
    gs_status st = check_common(mh, A, B, C, gather_to);
    if (st != GS_STATUS_SUCCESS) return st;
    uint32_t kernel = 0;
    st = gs_plan_gemm_strided_batched_ex(transa, transb, m, n, k, A[0], Atype, lda, strideA, B[0], Btype, ldb,
                                         strideB, C[0], Ctype, ldc, strideC, batchCount, computeType, &kernel);
    if (st != GS_STATUS_SUCCESS) return fail(mh, st, "invalid problem (gs_plan_gemm_strided_batched_ex)");
    const bool gather = gather_to != -1 && mh->ngpu > 1;
    if (gather && (ldc != m || (batchCount > 1 && strideC != static_cast<long long>(m) * n)))
        return fail(mh, GS_STATUS_NOT_SUPPORTED, "gather needs a dense C (ldc == m, strideC == m*n)");
    std::vector<long long> off(mh->ngpu + 1);
    gs_plan_shards(batchCount, mh->ngpu, 1, off.data());
    const size_t ea = elem_bytes(Atype), eb = elem_bytes(Btype), ec = elem_bytes(Ctype);
    const size_t mat_c = static_cast<size_t>(m) * n * ec;
    DeviceGuard guard;
    std::vector<int> active(mh->ngpu, 0);
    std::vector<size_t> c_off(mh->ngpu, 0), c_len(mh->ngpu, 0);
    for (int g = 0; g < mh->ngpu; ++g) {
        const long long lo = off[g], cnt = off[g + 1] - off[g];
        if (cnt <= 0) continue;
        cudaSetDevice(mh->devs[g]);
        cudaEventRecord(mh->ev0[g], mh->stream[g]);
        st = gs_gemm_strided_batched_ex(mh->h[g], transa, transb, m, n, k, alpha,
                                        static_cast<const char *>(A[g]) + lo * strideA * ea, Atype, lda, strideA,
                                        static_cast<const char *>(B[g]) + lo * strideB * eb, Btype, ldb, strideB, beta,
                                        static_cast<char *>(C[g]) + lo * strideC * ec, Ctype, ldc, strideC,
                                        static_cast<int>(cnt), computeType, algo);
        if (st != GS_STATUS_SUCCESS) {
            mh->last_error = std::string("device ") + std::to_string(mh->devs[g]) + ": " + gs_last_error(mh->h[g]);
            finish(mh, active, false);
            return st;
        }
        cudaEventRecord(mh->ev1[g], mh->stream[g]);
        active[g] = 1;
        c_off[g] = static_cast<size_t>(lo) * mat_c;
        c_len[g] = static_cast<size_t>(cnt) * mat_c;
    }
    if (gather) {
        st = gather_ranges(mh, C, c_off, c_len, gather_to);
        if (st != GS_STATUS_SUCCESS) {
            std::string why = mh->last_error;
            finish(mh, active, false);
            mh->last_error = why;
            return st;
        }
        for (int g = 0; g < mh->ngpu; ++g) {
            cudaSetDevice(mh->devs[g]);
            cudaEventRecord(mh->ev2[g], mh->stream[g]);
        }
    }
    return finish(mh, active, gather);
}

gs_status gs_gemm_batched_ex_multi(gs_multi_handle mh, int transa, int transb, int m, int n, int k,
                                   const void *alpha, const void *const *const Aarray[], int Atype, int lda,
                                   const void *const *const Barray[], int Btype, int ldb, const void *beta,
                                   void *const *const Carray[], int Ctype, int ldc, int batchCount, int computeType,
                                   int algo) {
    gs_status st = check_common(mh, Aarray, Barray, Carray, -1);
    if (st != GS_STATUS_SUCCESS) return st;
    if (batchCount < 0) return fail(mh, GS_STATUS_INVALID_VALUE, "batchCount < 0");
    std::vector<long long> off(mh->ngpu + 1);
    gs_plan_shards(batchCount, mh->ngpu, 1, off.data());
    DeviceGuard guard;
    std::vector<int> active(mh->ngpu, 0);
    for (int g = 0; g < mh->ngpu; ++g) {
        const long long lo = off[g], cnt = off[g + 1] - off[g];
        // batchCount == 0 still reaches device 0 so that argument errors surface as in gs_gemm_batched_ex.
        if (cnt <= 0 && !(batchCount == 0 && g == 0)) continue;
        cudaSetDevice(mh->devs[g]);
        cudaEventRecord(mh->ev0[g], mh->stream[g]);
        st = gs_gemm_batched_ex(mh->h[g], transa, transb, m, n, k, alpha, Aarray[g] + lo, Atype, lda, Barray[g] + lo,
                                Btype, ldb, beta, Carray[g] + lo, Ctype, ldc, static_cast<int>(cnt), computeType, algo);
        if (st != GS_STATUS_SUCCESS) {
            mh->last_error = std::string("device ") + std::to_string(mh->devs[g]) + ": " + gs_last_error(mh->h[g]);
            finish(mh, active, false);
            return st;
        }
        cudaEventRecord(mh->ev1[g], mh->stream[g]);
        active[g] = 1;
    }
    return finish(mh, active, false);
}

gs_status gs_gemm_ex_colsplit_multi(gs_multi_handle mh, int transa, int transb, int m, int n, int k,
                                    const void *alpha, const void *const A[], int Atype, int lda,
                                    const void *const B[], int Btype, int ldb, const void *beta, void *const C[],
                                    int Ctype, int ldc, int computeType, int algo, int gather_to) {
    gs_status st = check_common(mh, A, B, C, gather_to);
    if (st != GS_STATUS_SUCCESS) return st;
    uint32_t kernel = 0;
    st = gs_plan_gemm_strided_batched_ex(transa, transb, m, n, k, A[0], Atype, lda, 0, B[0], Btype, ldb, 0, C[0],
                                         Ctype, ldc, 0, 1, computeType, &kernel);
    if (st != GS_STATUS_SUCCESS) return fail(mh, st, "invalid problem (gs_plan_gemm_strided_batched_ex)");
    const bool gather = gather_to != -1 && mh->ngpu > 1;
    if (gather && ldc != m) return fail(mh, GS_STATUS_NOT_SUPPORTED, "gather needs a dense C (ldc == m)");
    std::vector<long long> off(mh->ngpu + 1);
    gs_plan_shards(n, mh->ngpu, GS_COLSPLIT_ALIGN, off.data());
    const size_t eb = elem_bytes(Btype), ec = elem_bytes(Ctype);
    DeviceGuard guard;
    std::vector<int> active(mh->ngpu, 0);
    std::vector<size_t> c_off(mh->ngpu, 0), c_len(mh->ngpu, 0);
    for (int g = 0; g < mh->ngpu; ++g) {
        const long long j0 = off[g], cols = off[g + 1] - off[g];
        if (cols <= 0 && !(n == 0 && g == 0)) continue;
        // Column j of op(B) is column j of B (op N) or row j of B (op T).
        const long long b_off = transb == GS_OP_N ? j0 * ldb : j0;
        cudaSetDevice(mh->devs[g]);
        cudaEventRecord(mh->ev0[g], mh->stream[g]);
        st = gs_gemm_ex(mh->h[g], transa, transb, m, static_cast<int>(cols), k, alpha, A[g], Atype, lda,
                        static_cast<const char *>(B[g]) + b_off * eb, Btype, ldb, beta,
                        static_cast<char *>(C[g]) + j0 * ldc * ec, Ctype, ldc, computeType, algo);
        if (st != GS_STATUS_SUCCESS) {
            mh->last_error = std::string("device ") + std::to_string(mh->devs[g]) + ": " + gs_last_error(mh->h[g]);
            finish(mh, active, false);
            return st;
        }
        cudaEventRecord(mh->ev1[g], mh->stream[g]);
        active[g] = 1;
        c_off[g] = static_cast<size_t>(j0) * ldc * ec;
        c_len[g] = static_cast<size_t>(cols) * ldc * ec;
    }
    if (gather) {
        st = gather_ranges(mh, C, c_off, c_len, gather_to);
        if (st != GS_STATUS_SUCCESS) {
            std::string why = mh->last_error;
            finish(mh, active, false);
            mh->last_error = why;
            return st;
        }
        for (int g = 0; g < mh->ngpu; ++g) {
            cudaSetDevice(mh->devs[g]);
            cudaEventRecord(mh->ev2[g], mh->stream[g]);
        }
    }
    return finish(mh, active, gather);
}

}  // extern "C"
