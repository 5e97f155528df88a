// gemm_simt.cu -- CUDA-core GEMM for operands the TMA path cannot address
// (leading dimensions, batch strides or base pointers that are not 16-byte
// aligned), and the k == 0 kernel that only applies beta.
//
// This is the B200 counterpart of slang-gemm's generic fallback shaders
// (shaders/gemm_lowp_f32.slang, shaders/gemm_integer_i32.slang): any op, any
// stride, f16/bf16/f32 inputs with f32 accumulation, s8 inputs with s32
// accumulation. It is a correctness path for unusual layouts, not a
// throughput path.
#include "gs_simt.cuh"

namespace gs {
namespace simt {

template <int IN, int OUT>
__global__ void __launch_bounds__(256) k_gemm_simt(const SimtArgs a) {
    __shared__ __align__(16) uint8_t smem[tile_smem_bytes<IN>()];
    grid_dep_wait();
    grid_dep_launch();
    simt_tiles<IN, OUT>(a, blockIdx.x, gridDim.x, smem);
}

// k == 0: every output is alpha*0 + beta*old.
template <int OUT>
__global__ void k_scale(const SimtArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const long long per = static_cast<long long>(a.m) * a.n;
    const long long total = per * a.batch;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(t / per);
        const long long r = t - b * per;
        const int gm = static_cast<int>(r % a.m), gn = static_cast<int>(r / a.m);
        void *Cb = a.c_arr ? a.c_arr[b]
                           : static_cast<uint8_t *>(a.C) + static_cast<size_t>(b) * a.stride_c * (OUT == OUT_F16 || OUT == OUT_BF16 ? 2 : 4);
        const size_t ci = static_cast<size_t>(gm) + static_cast<size_t>(gn) * a.ldc;
        if constexpr (OUT == OUT_I32) store_iacc(Cb, ci, 0, a.ep);
        else store_facc<OUT>(Cb, ci, 0.0f, a.ep);
    }
}

template <int IN, int OUT>
static cudaError_t go(Context &ctx, const SimtArgs &s) {
    const long long tiles = static_cast<long long>((s.m + TM - 1) / TM) * ((s.n + TN - 1) / TN) * s.batch;
    const long long cap = 16LL * (ctx.sm_count > 0 ? ctx.sm_count : 148);
    const dim3 grid(static_cast<unsigned>(tiles < cap ? tiles : cap));
    const cudaError_t e = launch_pdl(k_gemm_simt<IN, OUT>, grid, dim3(256), 0, ctx.stream, 1, s);
    ctx.launches++;
    return e;
}

static cudaError_t dispatch(Context &ctx, const GemmDesc &d, const SimtArgs &s) {
    if (d.in_kind == IN_F16 && d.out_kind == OUT_F32) return go<IN_F16, OUT_F32>(ctx, s);
    if (d.in_kind == IN_F16 && d.out_kind == OUT_F16) return go<IN_F16, OUT_F16>(ctx, s);
    if (d.in_kind == IN_BF16 && d.out_kind == OUT_F32) return go<IN_BF16, OUT_F32>(ctx, s);
    if (d.in_kind == IN_BF16 && d.out_kind == OUT_BF16) return go<IN_BF16, OUT_BF16>(ctx, s);
    if (d.in_kind == IN_I8 && d.out_kind == OUT_I32) return go<IN_I8, OUT_I32>(ctx, s);
    if (d.in_kind == IN_F32 && d.out_kind == OUT_F32) return go<IN_F32, OUT_F32>(ctx, s);
    return cudaErrorInvalidValue;
}

}  // namespace simt

cudaError_t launch_simt(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                        void *const *c_arr) {
    return simt::dispatch(ctx, d, simt::make_args(d, a_arr, b_arr, c_arr));
}

cudaError_t launch_scale(Context &ctx, const GemmDesc &d, void *const *c_arr) {
    using namespace simt;
    const SimtArgs s = make_args(d, nullptr, nullptr, c_arr);
    const long long total = static_cast<long long>(d.m) * d.n * d.batch;
    long long blocks = (total + 255) / 256;
    if (blocks > 4L * ctx.sm_count * 8) blocks = 4L * ctx.sm_count * 8;
    if (blocks < 1) blocks = 1;
    const dim3 grid(static_cast<unsigned>(blocks));
    cudaError_t e = cudaErrorInvalidValue;
    switch (d.out_kind) {
    case OUT_F32: e = launch_pdl(k_scale<OUT_F32>, grid, dim3(256), 0, ctx.stream, 1, s); break;
    case OUT_F16: e = launch_pdl(k_scale<OUT_F16>, grid, dim3(256), 0, ctx.stream, 1, s); break;
    case OUT_BF16: e = launch_pdl(k_scale<OUT_BF16>, grid, dim3(256), 0, ctx.stream, 1, s); break;
    case OUT_I32: e = launch_pdl(k_scale<OUT_I32>, grid, dim3(256), 0, ctx.stream, 1, s); break;
    }
    ctx.launches++;
    return e;
}

}  // namespace gs
