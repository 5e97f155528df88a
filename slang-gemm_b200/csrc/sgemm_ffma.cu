// sgemm_ffma.cu -- FP32 SGEMM on the CUDA cores (FFMA), column-major.
//
// Replaces slang-gemm's tiled FP32 shader (shaders/gemm_real_f32.slang) behind
// sgemm / sgemmStridedBatched (src/gemm.zig:286-317, :479-481). FP32 is not a
// reduced-precision contraction, so it stays on the FMA pipes.
//
// CTA tile 128 x 128, K step 8, 256 threads, 8 x 8 outputs per thread held in
// two 4x4 quadrants 64 rows / 64 columns apart (conflict-free float4 reads of
// the shared-memory panels). Shared memory is double buffered and the next
// K step's global loads are issued before the current step's FMAs. Interior
// tiles with 16-byte aligned operands use float4 global loads and stores;
// edge tiles and unaligned operands use guarded scalar accesses.
#include "gs_epilogue.cuh"
#include "gs_internal.h"

namespace gs {
namespace ffma {

constexpr int BM = 128, BN = 128, BK = 8;

struct FfmaArgs {
    int m, n, k, batch;
    const float *A; long long lda, stride_a;
    const float *B; long long ldb, stride_b;
    float *C; long long ldc, stride_c;
    int vec_a, vec_b, vec_c;  // operand allows float4 access along its contiguous dimension
    Epilogue ep;
};

// Loads this thread's 4 elements of the A panel (128 rows x 8 k) starting at k0.
//  op N: A[m + k*lda]  -> thread covers k = tid/32, m = (tid%32)*4 .. +3
//  op T: A[k + m*lda]  -> thread covers m = tid/2,  k = (tid%2)*4 .. +3
template <int TA>
__device__ __forceinline__ void load_a(const FfmaArgs &a, const float *A, int m0, int k0, int tid, bool fast, float (&r)[4]) {
    if constexpr (TA == 0) {
        const int kr = tid >> 5, mc = (tid & 31) * 4;
        const float *p = A + static_cast<size_t>(k0 + kr) * a.lda + m0 + mc;
        if (fast) {
            const float4 v = *reinterpret_cast<const float4 *>(p);
            r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) r[i] = (m0 + mc + i < a.m && k0 + kr < a.k) ? p[i] : 0.0f;
        }
    } else {
        const int mr = tid >> 1, kc = (tid & 1) * 4;
        const float *p = A + static_cast<size_t>(m0 + mr) * a.lda + k0 + kc;
        if (fast) {
            const float4 v = *reinterpret_cast<const float4 *>(p);
            r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) r[i] = (m0 + mr < a.m && k0 + kc + i < a.k) ? p[i] : 0.0f;
        }
    }
}

//  op N: B[k + n*ldb]  -> thread covers n = tid/2,  k = (tid%2)*4 .. +3
//  op T: B[n + k*ldb]  -> thread covers k = tid/32, n = (tid%32)*4 .. +3
template <int TB>
__device__ __forceinline__ void load_b(const FfmaArgs &a, const float *B, int n0, int k0, int tid, bool fast, float (&r)[4]) {
    if constexpr (TB == 0) {
        const int nr = tid >> 1, kc = (tid & 1) * 4;
        const float *p = B + static_cast<size_t>(n0 + nr) * a.ldb + k0 + kc;
        if (fast) {
            const float4 v = *reinterpret_cast<const float4 *>(p);
            r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) r[i] = (n0 + nr < a.n && k0 + kc + i < a.k) ? p[i] : 0.0f;
        }
    } else {
        const int kr = tid >> 5, nc = (tid & 31) * 4;
        const float *p = B + static_cast<size_t>(k0 + kr) * a.ldb + n0 + nc;
        if (fast) {
            const float4 v = *reinterpret_cast<const float4 *>(p);
            r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) r[i] = (n0 + nc + i < a.n && k0 + kr < a.k) ? p[i] : 0.0f;
        }
    }
}

template <int TA>
__device__ __forceinline__ void store_a(float (*As)[BM], int tid, const float (&r)[4]) {
    if constexpr (TA == 0) {
        const int kr = tid >> 5, mc = (tid & 31) * 4;
        *reinterpret_cast<float4 *>(&As[kr][mc]) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
        const int mr = tid >> 1, kc = (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) As[kc + i][mr] = r[i];
    }
}

template <int TB>
__device__ __forceinline__ void store_b(float (*Bs)[BN], int tid, const float (&r)[4]) {
    if constexpr (TB == 0) {
        const int nr = tid >> 1, kc = (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) Bs[kc + i][nr] = r[i];
    } else {
        const int kr = tid >> 5, nc = (tid & 31) * 4;
        *reinterpret_cast<float4 *>(&Bs[kr][nc]) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

template <int TA, int TB>
__global__ void __launch_bounds__(256, 2) k_sgemm_ffma(const FfmaArgs a) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const bool full_m = m0 + BM <= a.m, full_n = n0 + BN <= a.n;
    const int ktiles = (a.k + BK - 1) / BK;

    for (int b = blockIdx.z; b < a.batch; b += gridDim.z) {
        const float *A = a.A + static_cast<size_t>(b) * a.stride_a;
        const float *B = a.B + static_cast<size_t>(b) * a.stride_b;
        float *C = a.C + static_cast<size_t>(b) * a.stride_c;

        float acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

        float ra[4], rb[4];
        {
            const bool fk = BK <= a.k;
            load_a<TA>(a, A, m0, 0, tid, a.vec_a && full_m && fk, ra);
            load_b<TB>(a, B, n0, 0, tid, a.vec_b && full_n && fk, rb);
            store_a<TA>(As[0], tid, ra);
            store_b<TB>(Bs[0], tid, rb);
        }
        __syncthreads();

        for (int kt = 0; kt < ktiles; ++kt) {
            const int cur = kt & 1;
            const bool more = kt + 1 < ktiles;
            if (more) {
                const int k0 = (kt + 1) * BK;
                const bool fk = k0 + BK <= a.k;
                load_a<TA>(a, A, m0, k0, tid, a.vec_a && full_m && fk, ra);
                load_b<TB>(a, B, n0, k0, tid, a.vec_b && full_n && fk, rb);
            }
#pragma unroll
            for (int kk = 0; kk < BK; ++kk) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&As[cur][kk][tx * 4]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&As[cur][kk][64 + tx * 4]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][ty * 4]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[cur][kk][64 + ty * 4]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (more) {
                store_a<TA>(As[cur ^ 1], tid, ra);
                store_b<TB>(Bs[cur ^ 1], tid, rb);
            }
            __syncthreads();
        }

        // Epilogue: rows m0 + {tx*4 .. +3, 64 + tx*4 .. +3}, columns n0 + {ty*4 .. +3, 64 + ty*4 .. +3}.
        const bool fast_c = a.vec_c && full_m && full_n;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int gn = n0 + (j < 4 ? ty * 4 + j : 64 + ty * 4 + (j - 4));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int gm = m0 + h * 64 + tx * 4;
                float *p = C + static_cast<size_t>(gn) * a.ldc + gm;
                if (fast_c) {
                    float4 v = make_float4(acc[h * 4 + 0][j], acc[h * 4 + 1][j], acc[h * 4 + 2][j], acc[h * 4 + 3][j]);
                    if (!a.ep.identity) {
                        v.x *= a.ep.alpha_f; v.y *= a.ep.alpha_f; v.z *= a.ep.alpha_f; v.w *= a.ep.alpha_f;
                    }
                    if (!a.ep.beta_zero) {
                        const float4 o = *reinterpret_cast<const float4 *>(p);
                        v.x = __fadd_rn(v.x, __fmul_rn(a.ep.beta_f, o.x));
                        v.y = __fadd_rn(v.y, __fmul_rn(a.ep.beta_f, o.y));
                        v.z = __fadd_rn(v.z, __fmul_rn(a.ep.beta_f, o.z));
                        v.w = __fadd_rn(v.w, __fmul_rn(a.ep.beta_f, o.w));
                    }
                    *reinterpret_cast<float4 *>(p) = v;
                } else if (gn < a.n) {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (gm + i < a.m) store_facc<OUT_F32>(C, static_cast<size_t>(gn) * a.ldc + gm + i, acc[h * 4 + i][j], a.ep);
                }
            }
        }
    }
}

template <int TA, int TB>
static cudaError_t go(Context &ctx, const FfmaArgs &a) {
    dim3 grid((a.m + BM - 1) / BM, (a.n + BN - 1) / BN, a.batch < 65535 ? a.batch : 65535);
    k_sgemm_ffma<TA, TB><<<grid, 256, 0, ctx.stream>>>(a);
    ctx.launches++;
    return cudaGetLastError();
}

}  // namespace ffma

cudaError_t launch_ffma(Context &ctx, const GemmDesc &d) {
    using namespace ffma;
    FfmaArgs a{};
    a.m = d.m;
    a.n = d.n;
    a.k = d.k;
    a.batch = d.batch;
    a.A = static_cast<const float *>(d.A); a.lda = d.lda; a.stride_a = d.stride_a;
    a.B = static_cast<const float *>(d.B); a.ldb = d.ldb; a.stride_b = d.stride_b;
    a.C = static_cast<float *>(d.C); a.ldc = d.ldc; a.stride_c = d.stride_c;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const bool batched = d.batch > 1;
    a.vec_a = al16(d.A) && d.lda % 4 == 0 && (!batched || d.stride_a % 4 == 0);
    a.vec_b = al16(d.B) && d.ldb % 4 == 0 && (!batched || d.stride_b % 4 == 0);
    a.vec_c = al16(d.C) && d.ldc % 4 == 0 && (!batched || d.stride_c % 4 == 0);
    a.ep = d.ep;
    if (!d.trans_a && !d.trans_b) return go<0, 0>(ctx, a);
    if (!d.trans_a && d.trans_b) return go<0, 1>(ctx, a);
    if (d.trans_a && !d.trans_b) return go<1, 0>(ctx, a);
    return go<1, 1>(ctx, a);
}

}  // namespace gs
