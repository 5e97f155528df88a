// gemm_noalloc.cu -- gs_gemm_batched_ex_noalloc: the pointer-array batched
// GEMM for callers that cannot allocate device memory.
//
// Some callers own every byte of device memory themselves: a framework whose
// caching allocator holds the GPU's memory, a service that plans a fixed
// memory budget up front, or a latency-critical path that must not pay the
// device-wide synchronisation cudaMalloc and cudaFree can imply. They cannot
// create a gs_handle (gs_create allocates a small device word) and cannot let
// gs_gemm_batched_ex grow its tensor-map buffer. This entry point needs
// neither: the per-batch tensor maps, the misalignment flag and the device
// error word live in the file-scope array below, sized for at most
// GS_NOALLOC_MAX_BATCH batch entries. Every GPU that loads the library holds
// that array (3 * 256 tensor maps of 128 bytes plus 256 bytes of status words,
// 98,560 bytes) until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; each call clears the words that must start at zero. Calls whose
// work overlaps on the GPU (different streams, or different host threads)
// race on the array: order them on one stream. The array's device address is
// resolved once per device and kept for the life of the process, so the entry
// point must not be used on a device after cudaDeviceReset in that process
// (the reset unloads the module that holds the array).
#include <cstring>
#include <mutex>
#include <string>

#include "gs_internal.h"

namespace {

constexpr int kMaxBatch = GS_NOALLOC_MAX_BATCH;
constexpr size_t kMapBytes = 3ull * kMaxBatch * sizeof(CUtensorMap);  // A maps, B maps, C maps
constexpr size_t kWordBytes = 256;                                     // [0] error word, [1] / [2] misaligned flags
constexpr size_t kScratchBytes = kMapBytes + kWordBytes;
static_assert(sizeof(CUtensorMap) == 128 && kScratchBytes == 98560,
              "the size quoted in the comments and in include/gemm_sm100.h");

// Device scratch of the no-allocation path. In host code this name is only a
// stand-in for the symbol, never a device address: the kernels receive the
// address cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceSlot {
    void *scratch = nullptr;
    int sm_count = 0;
    bool ready = false;
};
DeviceSlot g_slots[64];
std::mutex g_slots_mu;

// Set-up, once per device, with that device current: resolve the device
// address of the scratch array and the SM count. No allocation.
gs_status device_slot(int dev, DeviceSlot **out) {
    if (dev < 0 || dev >= 64) return GS_STATUS_NOT_SUPPORTED;
    std::lock_guard<std::mutex> lock(g_slots_mu);
    DeviceSlot &s = g_slots[dev];
    if (!s.ready) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return GS_STATUS_NOT_INITIALIZED;
        }
        if (major != 10 || minor != 0) return GS_STATUS_ARCH_MISMATCH;
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
            cudaGetLastError();
            return GS_STATUS_EXECUTION_FAILED;
        }
        s.scratch = ptr;
        s.sm_count = sms;
        s.ready = true;
    }
    *out = &s;
    return GS_STATUS_SUCCESS;
}

}  // namespace

extern "C" gs_status gs_gemm_batched_ex_noalloc(void *stream, int transa, int transb, int m, int n, int k,
                                                const void *alpha, const void *const Aarray[], int Atype, int lda,
                                                const void *const Barray[], int Btype, int ldb, const void *beta,
                                                void *const Carray[], int Ctype, int ldc, int batchCount,
                                                int computeType) {
    using namespace gs;
    GemmDesc d{};
    std::string why;
    gs_status st = check_shape_core(transa, transb, m, n, k, lda, ldb, ldc, batchCount, &d, &why);
    if (st != GS_STATUS_SUCCESS) return st;
    TypedArgs t;
    st = decode_types(Atype, Btype, Ctype, computeType, &t);
    if (st != GS_STATUS_SUCCESS) return st;
    if (t.in == IN_I8 && k > 131071) return GS_STATUS_NOT_SUPPORTED;
    if (batchCount > kMaxBatch) return GS_STATUS_INVALID_VALUE;  // beyond the static scratch
    if (!alpha || !beta) return GS_STATUS_INVALID_VALUE;
    if (m == 0 || n == 0 || batchCount == 0) return GS_STATUS_SUCCESS;
    if (!Carray || (k > 0 && (!Aarray || !Barray))) return GS_STATUS_INVALID_VALUE;

    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    DeviceSlot *slot = nullptr;
    st = device_slot(dev, &slot);
    if (st != GS_STATUS_SUCCESS) return st;

    // A context over the static scratch: nothing in it owns device memory.
    Context ctx;
    ctx.device = dev;
    ctx.sm_count = slot->sm_count;
    ctx.stream = static_cast<cudaStream_t>(stream);
    ctx.may_allocate = false;
    ctx.tmap_buf = slot->scratch;
    ctx.tmap_bytes = kMapBytes;
    ctx.dev_err = reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(slot->scratch) + kMapBytes);
    cudaError_t e = cudaMemsetAsync(ctx.dev_err, 0, 3 * sizeof(uint32_t), ctx.stream);
    if (e == cudaSuccess) {
        d.in_kind = t.in;
        d.out_kind = t.out;
        d.algo = GS_GEMM_DEFAULT;
        read_scalars(computeType, alpha, beta, &d.ep);
        const long long es = static_cast<long long>(in_elem_size(t.in));
        if (k == 0) {
            e = launch_scale(ctx, d, Carray);
        } else if (t.in != IN_F32 && (d.lda * es) % 16 == 0 && (d.ldb * es) % 16 == 0) {
            e = launch_tc_ptr_array(ctx, d, Aarray, Barray, Carray);
        } else if (t.in == IN_F32) {
            e = launch_ffma_ptr(ctx, d, Aarray, Barray, Carray);
        } else {
            e = launch_simt(ctx, d, Aarray, Barray, Carray);
        }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_EXECUTION_FAILED;
    }
    return GS_STATUS_SUCCESS;
}

extern "C" gs_status gs_noalloc_device_error(void *stream, uint32_t *word) {
    using namespace gs;
    if (!word) return GS_STATUS_INVALID_VALUE;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_NOT_INITIALIZED;
    }
    DeviceSlot *slot = nullptr;
    gs_status st = device_slot(dev, &slot);
    if (st != GS_STATUS_SUCCESS) return st;
    // The word sits right after the tensor maps; a plain device-to-host copy of 4 bytes, no allocation.
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess ||
        cudaMemcpy(word, static_cast<unsigned char *>(slot->scratch) + kMapBytes, sizeof(uint32_t),
                   cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return GS_STATUS_EXECUTION_FAILED;
    }
    return GS_STATUS_SUCCESS;
}
