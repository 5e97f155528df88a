// gemm_simt.cu -- CUDA-core GEMM for operands the TMA path cannot address
// (leading dimensions, batch strides or base pointers that are not 16-byte
// aligned), and the k == 0 kernel that only applies beta.
//
// This is the B200 counterpart of slang-gemm's generic fallback shaders
// (shaders/gemm_lowp_f32.slang, shaders/gemm_integer_i32.slang): any op, any
// stride, f16/bf16/f32 inputs with f32 accumulation, s8 inputs with s32
// accumulation. It is a correctness path for unusual layouts, not a
// throughput path.
#include "gs_epilogue.cuh"
#include "gs_internal.h"

namespace gs {
namespace simt {

constexpr int TM = 64, TN = 64, TK = 16;

struct SimtArgs {
    int trans_a, trans_b;
    int m, n, k, batch;
    const void *A; long long lda, stride_a;
    const void *B; long long ldb, stride_b;
    void *C; long long ldc, stride_c;
    const void *const *a_arr;
    const void *const *b_arr;
    void *const *c_arr;
    const uint32_t *run_flag;  // when set: do the work only if *run_flag == run_gen
    uint32_t run_gen;
    Epilogue ep;
};

template <int IN>
__device__ __forceinline__ auto load_elem(const void *p, size_t i) {
    if constexpr (IN == IN_F16) return __half2float(static_cast<const __half *>(p)[i]);
    else if constexpr (IN == IN_BF16) return bf16_bits_to_f32(static_cast<const uint16_t *>(p)[i]);
    else if constexpr (IN == IN_F32) return static_cast<const float *>(p)[i];
    else return static_cast<int32_t>(static_cast<const int8_t *>(p)[i]);
}

template <int IN, int OUT>
__global__ void __launch_bounds__(256) k_gemm_simt(const SimtArgs a) {
    using Acc = typename std::conditional<IN == IN_I8, int32_t, float>::type;
    __shared__ Acc As[TK][TM];
    __shared__ Acc Bs[TK][TN + 1];
    grid_dep_wait();
    grid_dep_launch();
    if (a.run_flag != nullptr && *a.run_flag != a.run_gen) return;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.x * TM, n0 = blockIdx.y * TN;
    for (int b = blockIdx.z; b < a.batch; b += gridDim.z) {
        const void *Ab = a.a_arr ? a.a_arr[b]
                                 : static_cast<const uint8_t *>(a.A) + static_cast<size_t>(b) * a.stride_a * (IN == IN_I8 ? 1 : (IN == IN_F32 ? 4 : 2));
        const void *Bb = a.b_arr ? a.b_arr[b]
                                 : static_cast<const uint8_t *>(a.B) + static_cast<size_t>(b) * a.stride_b * (IN == IN_I8 ? 1 : (IN == IN_F32 ? 4 : 2));
        void *Cb = a.c_arr ? a.c_arr[b]
                           : static_cast<uint8_t *>(a.C) + static_cast<size_t>(b) * a.stride_c * (OUT == OUT_F16 || OUT == OUT_BF16 ? 2 : 4);
        Acc acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = Acc(0);
        for (int k0 = 0; k0 < a.k; k0 += TK) {
            // 64x16 A elements and 16x64 B elements, 4 of each per thread.
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int idx = tid + e * 256;
                const int mm = idx % TM, kk = idx / TM;
                const int gm = m0 + mm, gk = k0 + kk;
                Acc v = Acc(0);
                if (gm < a.m && gk < a.k) {
                    const size_t off = a.trans_a ? static_cast<size_t>(gk) + static_cast<size_t>(gm) * a.lda
                                                 : static_cast<size_t>(gm) + static_cast<size_t>(gk) * a.lda;
                    v = static_cast<Acc>(load_elem<IN>(Ab, off));
                }
                As[kk][mm] = v;
                const int nn = idx % TN, kb = idx / TN;
                const int gn = n0 + nn, gk2 = k0 + kb;
                Acc w = Acc(0);
                if (gn < a.n && gk2 < a.k) {
                    const size_t off = a.trans_b ? static_cast<size_t>(gn) + static_cast<size_t>(gk2) * a.ldb
                                                 : static_cast<size_t>(gk2) + static_cast<size_t>(gn) * a.ldb;
                    w = static_cast<Acc>(load_elem<IN>(Bb, off));
                }
                Bs[kb][nn] = w;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < TK; ++kk) {
                Acc av[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = As[kk][tx + 16 * i];
#pragma unroll
                for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][ty + 16 * j];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int gm = m0 + tx + 16 * i;
            if (gm >= a.m) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int gn = n0 + ty + 16 * j;
                if (gn >= a.n) continue;
                const size_t ci = static_cast<size_t>(gm) + static_cast<size_t>(gn) * a.ldc;
                if constexpr (OUT == OUT_I32) store_iacc(Cb, ci, acc[i][j], a.ep);
                else store_facc<OUT>(Cb, ci, acc[i][j], a.ep);
            }
        }
    }
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

static SimtArgs make_args(const GemmDesc &d, const void *const *a_arr, const void *const *b_arr, void *const *c_arr,
                          const uint32_t *flag, uint32_t gen) {
    SimtArgs s{};
    s.trans_a = d.trans_a;
    s.trans_b = d.trans_b;
    s.m = d.m;
    s.n = d.n;
    s.k = d.k;
    s.batch = d.batch;
    s.A = d.A; s.lda = d.lda; s.stride_a = d.stride_a;
    s.B = d.B; s.ldb = d.ldb; s.stride_b = d.stride_b;
    s.C = d.C; s.ldc = d.ldc; s.stride_c = d.stride_c;
    s.a_arr = a_arr;
    s.b_arr = b_arr;
    s.c_arr = c_arr;
    s.run_flag = flag;
    s.run_gen = gen;
    s.ep = d.ep;
    return s;
}

template <int IN, int OUT>
static cudaError_t go(Context &ctx, const SimtArgs &s) {
    dim3 grid((s.m + TM - 1) / TM, (s.n + TN - 1) / TN, s.batch < 65535 ? s.batch : 65535);
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
    return simt::dispatch(ctx, d, simt::make_args(d, a_arr, b_arr, c_arr, nullptr, 0u));
}

cudaError_t launch_simt_if_flag(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                                void *const *c_arr, const uint32_t *flag, uint32_t gen) {
    return simt::dispatch(ctx, d, simt::make_args(d, a_arr, b_arr, c_arr, flag, gen));
}

cudaError_t launch_scale(Context &ctx, const GemmDesc &d, void *const *c_arr) {
    using namespace simt;
    const SimtArgs s = make_args(d, nullptr, nullptr, c_arr, nullptr, 0u);
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
