// gs_internal.h -- shared declarations between the C-ABI layer and the kernels.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/gemm_sm100.h"

namespace gs {

// Element / output kinds the kernels are specialised on.
// IN_TF32: fp32 storage read by tcgen05 kind::tf32 (the operands the FAST_TF32
// path prepares, each value split into two tf32-exact parts).
enum InKind { IN_F16 = 0, IN_BF16 = 1, IN_I8 = 2, IN_F32 = 3, IN_TF32 = 4 };
enum OutKind { OUT_F32 = 0, OUT_I32 = 1, OUT_F16 = 2, OUT_BF16 = 3 };

// Epilogue scalars. Which fields are used depends on the output / compute kind.
struct Epilogue {
    float alpha_f, beta_f;    // f32 compute (16F compute is widened to f32)
    int32_t alpha_i, beta_i;  // 32I compute
    int beta_zero;            // beta == 0: C is not read
    int identity;             // alpha == 1 and beta == 0: store the accumulator as is
};

// One (possibly batched) GEMM as the kernels see it, column-major, after the
// C-ABI layer has validated it. Pointers are device pointers.
struct GemmDesc {
    int trans_a, trans_b;     // 0 = N, 1 = T (C is folded into T for real types)
    int m, n, k;
    int batch;
    InKind in_kind;
    OutKind out_kind;
    const void *A; long long lda, stride_a;
    const void *B; long long ldb, stride_b;
    void *C; long long ldc, stride_c;
    Epilogue ep;
    int algo;                 // cublasGemmAlgo_t hint: 0 = 1-SM tile, 1 = 2-SM pair tile, else automatic
    int fast_tf32;            // COMPUTE_32F_FAST_TF32 on f32 operands: TF32 tensor-core products allowed
};

// Kernel selection made by plan_gemm (pure host logic, no device calls).
struct Plan {
    uint32_t kernel;          // one GS_KERNEL_* bit
};

// Host-side context behind gs_handle.
// Default limit of the kernels' bounded waits: 4e9 SM cycles, about 2 s at the
// B200's 1.965 GHz top clock; any legitimate wait in these kernels is far shorter.
constexpr long long kDefaultWaitLimitCycles = 4000000000LL;

struct Context {
    int device = -1;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    uint32_t *dev_err = nullptr;      // [0] error word of bounded waits, [1] / [2] pointer-array A,B / C misalignment flags
    long long spin_limit = kDefaultWaitLimitCycles;  // SM cycles after which a bounded wait gives up
    int debug_skip_kb = -1;           // test hook of gs_debug_skip_kblock (-1 = off)
    uint32_t last_kernels = 0;
    uint64_t launches = 0;
    std::string last_error;
    // staging buffers of the host-buffer mirror (gs_host_gemm_ex)
    void *stage = nullptr;
    size_t stage_bytes = 0;
    // copy streams and events of the pipelined host-buffer mirror (created on first use)
    cudaStream_t h2d = nullptr, d2h = nullptr;
    static constexpr int kMaxChunks = 32;
    cudaEvent_t ev_start = nullptr, ev_a = nullptr;
    cudaEvent_t ev_in[kMaxChunks] = {}, ev_out[kMaxChunks] = {};
    // device copy of tensor maps for pointer-array batches; buffers it outgrew are freed with the handle
    void *tmap_buf = nullptr;
    size_t tmap_bytes = 0;
    std::vector<void *> retired;
    // stream-K workspace of the FP32 FFMA kernel: two partial tiles per resident CTA, and per-tile counters
    void *sk_buf = nullptr;
    size_t sk_bytes = 0;
    void *sk_counts = nullptr;
    size_t sk_count_bytes = 0;
    // split-K workspace of the tensor-core path: one f32 / s32 partial C per K slice
    void *splitk_buf = nullptr;
    size_t splitk_bytes = 0;
    // false for contexts over caller-provided memory only (the no-allocation entry point)
    bool may_allocate = true;
    // split operands of the FAST_TF32 tensor-core path
    void *tf32_buf = nullptr;
    size_t tf32_bytes = 0;
    // Pointer-array calls tag the misalignment word with a per-call value
    // instead of clearing it first (one stream operation less per call).
    uint32_t ptr_gen = 0;
    uint32_t next_ptr_gen() {
        if (++ptr_gen == 0) ++ptr_gen;
        return ptr_gen;
    }
};

// Programmatic dependent launch: every kernel of this library starts with
// griddepcontrol.wait (before touching global memory) and then lets its own
// dependents be scheduled, so each launch may be issued before the previous
// kernel in the stream has finished; the GPU overlaps the launch latency.
#ifdef __CUDACC__
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
    if (cluster > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = static_cast<unsigned>(n);
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

// Validation + kernel choice for a strided (or single) GEMM; no device calls.
gs_status plan_gemm(const GemmDesc &d, Plan *plan, std::string *why);

// Launchers (return cudaSuccess or the launch error).
cudaError_t launch_tc(Context &ctx, const GemmDesc &d);
// Tile (1 = 1-SM 128x256, 2 = pair 256x256, 3 = wide 256x512) and K slices a tensor-core call would use.
void plan_tc_tile(const GemmDesc &d, int sm_count, int *tile, int *k_slices);
// FAST_TF32 f32 GEMM on the tensor cores: splits A and B into tf32-exact
// high/low parts and runs one kind::tf32 GEMM over the concatenated K.
cudaError_t launch_tf32(Context &ctx, const GemmDesc &d);
// Whether a FAST_TF32 problem is large enough for the tensor-core path to win.
bool tf32_worthwhile(const GemmDesc &d);
cudaError_t launch_tc_ptr_array(Context &ctx, const GemmDesc &d, const void *const *a_arr,
                                const void *const *b_arr, void *const *c_arr);
cudaError_t launch_ffma(Context &ctx, const GemmDesc &d);
cudaError_t launch_ffma_ptr(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                            void *const *c_arr);
cudaError_t launch_simt(Context &ctx, const GemmDesc &d, const void *const *a_arr,
                        const void *const *b_arr, void *const *c_arr);
cudaError_t launch_scale(Context &ctx, const GemmDesc &d, void *const *c_arr);

// Tensor-map encoder obtained from the driver at run time.
bool encode_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t dim0,
                    uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                    uint32_t box0, uint32_t box1, std::string *why,
                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

size_t in_elem_size(InKind k);
size_t out_elem_size(OutKind k);

// Argument decoding shared by the C entry points (capi.cu).
struct TypedArgs {
    InKind in;
    OutKind out;
};
gs_status decode_types(int at, int bt, int ct, int comp, TypedArgs *t);
void read_scalars(int comp, const void *alpha, const void *beta, Epilogue *ep);
gs_status check_shape_core(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int batch,
                           GemmDesc *d, std::string *why);

}  // namespace gs

// The object behind gs_handle.
struct gs_context {
    gs::Context ctx;
};
