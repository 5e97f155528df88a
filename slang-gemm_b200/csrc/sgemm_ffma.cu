// sgemm_ffma.cu -- FP32 SGEMM on the CUDA cores (FFMA), column-major.
//
// Replaces slang-gemm's tiled FP32 shader (shaders/gemm_real_f32.slang) behind
// sgemm / sgemmStridedBatched (src/gemm.zig:286-317, :479-481). FP32 is not a
// reduced-precision contraction, so it stays on the FMA pipes.
//
// One kernel template, three CTA tiles chosen by problem size so that the grid
// fills the 148 SMs:
//   128 x 128 (256 threads, 8 x 8 outputs per thread, 2 CTAs per SM)  large
//    64 x  64 (128 threads, 4 x 8, 4 CTAs per SM)                      medium
//    32 x  32 ( 64 threads, 4 x 4)                                     small
// K step 16. The FMAs are Blackwell's packed FP32 FMA (FFMA2, __ffma2_rn):
// one instruction updates two rows of an output column, which halves the
// FMA instruction count — a kernel issuing one FFMA per cycle per scheduler is
// issue-bound below the FMA pipe's rate, the packed form is not. Each thread's outputs are 4 x 4 blocks spaced BM/2 (BN/2) apart
// when it holds 8 rows (columns), so its shared-memory reads are conflict-free
// float4 loads. Shared memory is double buffered; the next K step's global
// loads are issued before the current step's FMAs and stored after them, and
// the operand fragments of step kk+1 are read from shared memory while step
// kk's FMAs run. Interior tiles of 16-byte aligned operands use float4 global
// loads and stores; edge tiles and unaligned operands use guarded scalar
// accesses. Operands stored K-contiguous (A op T, B op N) are transposed into
// the [k][m] / [k][n] shared layout with scalar stores into rows padded by 4
// floats (at most 2-way bank conflicts).
//
// Problems whose 64 x 64 grid cannot fill the SMs (512^3 gives 64 tiles) split
// K across a thread-block cluster of S CTAs (S = 2, 4, 8): each CTA runs the
// same tile over 1/S of the K steps, parks its partial tile in shared memory,
// and after a cluster barrier CTA r sums slice r of the tile from all S
// partials through distributed shared memory, in rank order (deterministic),
// and applies alpha / beta. No workspace, no atomics, one launch.
#include <cooperative_groups.h>

#include "gs_epilogue.cuh"
#include "gs_internal.h"

namespace gs {
namespace ffma {

struct FfmaArgs {
    int m, n, k, batch;
    const float *A; long long lda, stride_a;
    const float *B; long long ldb, stride_b;
    float *C; long long ldc, stride_c;
    int vec_a, vec_b, vec_c;  // leading dimension / stride allow float4 access along the contiguous dimension
    const float *const *a_arr;  // pointer-array batches (else nullptr): per-entry A, B, C
    const float *const *b_arr;
    float *const *c_arr;
    Epilogue ep;
};

template <int BM_, int BN_, int TM_, int TN_, int MINB_, int BK_ = 16>
struct Tile {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_, MINB = MINB_;
    static constexpr int TX = BM / TM, TY = BN / TN;        // threads along M and N
    static constexpr int THREADS = TX * TY;
    static constexpr int RM = TM / 4, RN = TN / 4;          // 4 x 4 blocks per thread along M and N
    static constexpr int CH_A = BM * BK / 4 / THREADS;      // float4 chunks of A per thread per K step
    static constexpr int CH_B = BN * BK / 4 / THREADS;
    static_assert(CH_A * THREADS * 4 == BM * BK && CH_B * THREADS * 4 == BN * BK, "tile / thread mismatch");
};
using TileL = Tile<128, 128, 8, 8, 2>;
using TileM = Tile<64, 64, 4, 8, 4>;
using TileS = Tile<32, 32, 4, 4, 4>;

// Chunk c of the A tile (BM rows x BK k) as (row or k, offset) for the stored layout.
//  op N (M-contiguous): c -> k = c / (BM/4), m = (c % (BM/4)) * 4 .. +3
//  op T (K-contiguous): c -> m = c / (BK/4), k = (c % (BK/4)) * 4 .. +3
template <int TA, class T>
__device__ __forceinline__ void load_a(const FfmaArgs &a, const float *A, int m0, int k0, int c, bool fast, float4 &r) {
    if constexpr (TA == 0) {
        const int kr = c / (T::BM / 4), mc = (c % (T::BM / 4)) * 4;
        const float *p = A + static_cast<size_t>(k0 + kr) * a.lda + m0 + mc;
        if (fast) {
            r = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
            const bool kin = k0 + kr < a.k;
            r.x = (kin && m0 + mc + 0 < a.m) ? p[0] : 0.0f;
            r.y = (kin && m0 + mc + 1 < a.m) ? p[1] : 0.0f;
            r.z = (kin && m0 + mc + 2 < a.m) ? p[2] : 0.0f;
            r.w = (kin && m0 + mc + 3 < a.m) ? p[3] : 0.0f;
        }
    } else {
        const int mr = c / (T::BK / 4), kc = (c % (T::BK / 4)) * 4;
        const float *p = A + static_cast<size_t>(m0 + mr) * a.lda + k0 + kc;
        if (fast) {
            r = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
            const bool min_ = m0 + mr < a.m;
            r.x = (min_ && k0 + kc + 0 < a.k) ? p[0] : 0.0f;
            r.y = (min_ && k0 + kc + 1 < a.k) ? p[1] : 0.0f;
            r.z = (min_ && k0 + kc + 2 < a.k) ? p[2] : 0.0f;
            r.w = (min_ && k0 + kc + 3 < a.k) ? p[3] : 0.0f;
        }
    }
}

//  op N (K-contiguous): c -> n = c / (BK/4), k = (c % (BK/4)) * 4 .. +3
//  op T (N-contiguous): c -> k = c / (BN/4), n = (c % (BN/4)) * 4 .. +3
template <int TB, class T>
__device__ __forceinline__ void load_b(const FfmaArgs &a, const float *B, int n0, int k0, int c, bool fast, float4 &r) {
    if constexpr (TB == 0) {
        const int nr = c / (T::BK / 4), kc = (c % (T::BK / 4)) * 4;
        const float *p = B + static_cast<size_t>(n0 + nr) * a.ldb + k0 + kc;
        if (fast) {
            r = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
            const bool nin = n0 + nr < a.n;
            r.x = (nin && k0 + kc + 0 < a.k) ? p[0] : 0.0f;
            r.y = (nin && k0 + kc + 1 < a.k) ? p[1] : 0.0f;
            r.z = (nin && k0 + kc + 2 < a.k) ? p[2] : 0.0f;
            r.w = (nin && k0 + kc + 3 < a.k) ? p[3] : 0.0f;
        }
    } else {
        const int kr = c / (T::BN / 4), nc = (c % (T::BN / 4)) * 4;
        const float *p = B + static_cast<size_t>(k0 + kr) * a.ldb + n0 + nc;
        if (fast) {
            r = __ldg(reinterpret_cast<const float4 *>(p));
        } else {
            const bool kin = k0 + kr < a.k;
            r.x = (kin && n0 + nc + 0 < a.n) ? p[0] : 0.0f;
            r.y = (kin && n0 + nc + 1 < a.n) ? p[1] : 0.0f;
            r.z = (kin && n0 + nc + 2 < a.n) ? p[2] : 0.0f;
            r.w = (kin && n0 + nc + 3 < a.n) ? p[3] : 0.0f;
        }
    }
}

// Shared layouts: As[k][m] with row length LDA_S, Bs[k][n] with row length LDB_S.
template <int TA, class T>
__device__ __forceinline__ void store_a(float *As, int lds, int c, const float4 &r) {
    if constexpr (TA == 0) {
        const int kr = c / (T::BM / 4), mc = (c % (T::BM / 4)) * 4;
        *reinterpret_cast<float4 *>(&As[kr * lds + mc]) = r;
    } else {
        const int mr = c / (T::BK / 4), kc = (c % (T::BK / 4)) * 4;
        As[(kc + 0) * lds + mr] = r.x;
        As[(kc + 1) * lds + mr] = r.y;
        As[(kc + 2) * lds + mr] = r.z;
        As[(kc + 3) * lds + mr] = r.w;
    }
}

template <int TB, class T>
__device__ __forceinline__ void store_b(float *Bs, int lds, int c, const float4 &r) {
    if constexpr (TB == 0) {
        const int nr = c / (T::BK / 4), kc = (c % (T::BK / 4)) * 4;
        Bs[(kc + 0) * lds + nr] = r.x;
        Bs[(kc + 1) * lds + nr] = r.y;
        Bs[(kc + 2) * lds + nr] = r.z;
        Bs[(kc + 3) * lds + nr] = r.w;
    } else {
        const int kr = c / (T::BN / 4), nc = (c % (T::BN / 4)) * 4;
        *reinterpret_cast<float4 *>(&Bs[kr * lds + nc]) = r;
    }
}

// alpha * v then + beta * C, four consecutive rows of one column (16-byte aligned).
__device__ __forceinline__ void store4(float *p, float4 v, const Epilogue &ep) {
    if (!ep.identity) {
        v.x = __fmul_rn(ep.alpha_f, v.x); v.y = __fmul_rn(ep.alpha_f, v.y);
        v.z = __fmul_rn(ep.alpha_f, v.z); v.w = __fmul_rn(ep.alpha_f, v.w);
    }
    if (!ep.beta_zero) {
        const float4 o = *reinterpret_cast<const float4 *>(p);
        v.x = __fadd_rn(v.x, __fmul_rn(ep.beta_f, o.x));
        v.y = __fadd_rn(v.y, __fmul_rn(ep.beta_f, o.y));
        v.z = __fadd_rn(v.z, __fmul_rn(ep.beta_f, o.z));
        v.w = __fadd_rn(v.w, __fmul_rn(ep.beta_f, o.w));
    }
    *reinterpret_cast<float4 *>(p) = v;
}

// Row lengths of the shared-memory operand tiles (As[k][m], Bs[k][n], double buffered); rows are padded
// when they are filled by transposing stores.
template <int TA, int TB, class T>
struct Smem {
    static constexpr int LDA_S = T::BM + (TA == 1 ? 4 : 0);
    static constexpr int LDB_S = T::BN + (TB == 0 ? 4 : 0);
};

// Accumulates op(A)[m0.., k] x op(B)[k, n0..] over the K steps [kt0, kt1) of one tile into acc2
// (acc2[ip][j] = rows 2ip, 2ip+1 of this thread, column j). Starts and ends with the CTA synchronised, so
// the shared tiles are free again when it returns. Used by the stream-K kernel; the data-parallel kernel
// below keeps the same loop written inline, where ptxas allocates it fewer registers (4-12 bytes of spill
// for the 128 x 128 tile instead of 60-104 through this function, -Xptxas -v).
template <int TA, int TB, class T>
__device__ __forceinline__ void k_loop(const FfmaArgs &a, const float *A, const float *B, int m0, int n0, int kt0,
                                       int kt1, bool va, bool vb,
                                       float (&As)[2][T::BK * Smem<TA, TB, T>::LDA_S],
                                       float (&Bs)[2][T::BK * Smem<TA, TB, T>::LDB_S],
                                       float2 (&acc2)[2 * T::RM][4 * T::RN]) {
    constexpr int BM = T::BM, BN = T::BN, BK = T::BK, RM = T::RM, RN = T::RN;
    constexpr int LDA_S = Smem<TA, TB, T>::LDA_S, LDB_S = Smem<TA, TB, T>::LDB_S;
    const int tid = threadIdx.x;
    const int tx = tid % T::TX, ty = tid / T::TX;
    const bool full_m = m0 + BM <= a.m, full_n = n0 + BN <= a.n;
    float4 ra[T::CH_A], rb[T::CH_B];
    if (kt0 < kt1) {
        const int k0 = kt0 * BK;
        const bool fk = k0 + BK <= a.k;
#pragma unroll
        for (int i = 0; i < T::CH_A; ++i) load_a<TA, T>(a, A, m0, k0, tid + i * T::THREADS, va && full_m && fk, ra[i]);
#pragma unroll
        for (int i = 0; i < T::CH_B; ++i) load_b<TB, T>(a, B, n0, k0, tid + i * T::THREADS, vb && full_n && fk, rb[i]);
#pragma unroll
        for (int i = 0; i < T::CH_A; ++i) store_a<TA, T>(As[0], LDA_S, tid + i * T::THREADS, ra[i]);
#pragma unroll
        for (int i = 0; i < T::CH_B; ++i) store_b<TB, T>(Bs[0], LDB_S, tid + i * T::THREADS, rb[i]);
    }
    __syncthreads();

    for (int kt = kt0; kt < kt1; ++kt) {
        const int cur = (kt - kt0) & 1;
        const bool more = kt + 1 < kt1;
        if (more) {
            const int k0 = (kt + 1) * BK;
            const bool fk = k0 + BK <= a.k;
#pragma unroll
            for (int i = 0; i < T::CH_A; ++i)
                load_a<TA, T>(a, A, m0, k0, tid + i * T::THREADS, va && full_m && fk, ra[i]);
#pragma unroll
            for (int i = 0; i < T::CH_B; ++i)
                load_b<TB, T>(a, B, n0, k0, tid + i * T::THREADS, vb && full_n && fk, rb[i]);
        }
        const float *as = As[cur];
        const float *bs = Bs[cur];
        float4 fa[2][RM], fb[2][RN];
#pragma unroll
        for (int r = 0; r < RM; ++r) fa[0][r] = *reinterpret_cast<const float4 *>(&as[r * (BM / RM) + tx * 4]);
#pragma unroll
        for (int r = 0; r < RN; ++r) fb[0][r] = *reinterpret_cast<const float4 *>(&bs[r * (BN / RN) + ty * 4]);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const int f = kk & 1;
            if (kk + 1 < BK) {
#pragma unroll
                for (int r = 0; r < RM; ++r)
                    fa[f ^ 1][r] = *reinterpret_cast<const float4 *>(&as[(kk + 1) * LDA_S + r * (BM / RM) + tx * 4]);
#pragma unroll
                for (int r = 0; r < RN; ++r)
                    fb[f ^ 1][r] = *reinterpret_cast<const float4 *>(&bs[(kk + 1) * LDB_S + r * (BN / RN) + ty * 4]);
            }
            // Packed FP32 FMA (FFMA2): two rows of one output column per instruction, each
            // element rounded once exactly as fmaf rounds it.
#pragma unroll
            for (int j = 0; j < 4 * RN; ++j) {
                const float4 &vbv = fb[f][j / 4];
                const float bv = (j & 3) == 0 ? vbv.x : (j & 3) == 1 ? vbv.y : (j & 3) == 2 ? vbv.z : vbv.w;
                const float2 b2 = make_float2(bv, bv);
#pragma unroll
                for (int ip = 0; ip < 2 * RM; ++ip) {
                    const float4 &vav = fa[f][ip / 2];
                    const float2 a2 = (ip & 1) ? make_float2(vav.z, vav.w) : make_float2(vav.x, vav.y);
                    acc2[ip][j] = __ffma2_rn(a2, b2, acc2[ip][j]);
                }
            }
        }
        if (more) {
#pragma unroll
            for (int i = 0; i < T::CH_A; ++i) store_a<TA, T>(As[cur ^ 1], LDA_S, tid + i * T::THREADS, ra[i]);
#pragma unroll
            for (int i = 0; i < T::CH_B; ++i) store_b<TB, T>(Bs[cur ^ 1], LDB_S, tid + i * T::THREADS, rb[i]);
        }
        __syncthreads();
    }
}

// Writes a finished tile: rows m0 + r*(BM/RM) + tx*4 + {0..3}, columns n0 + s*(BN/RN) + ty*4 + {0..3};
// alpha*acc then + beta*C with separate roundings, as gemm(f32) does (src/gemm.zig:523-544).
template <class T>
__device__ __forceinline__ void store_tile(const FfmaArgs &a, float *C, int m0, int n0, bool vc,
                                           const float2 (&acc2)[2 * T::RM][4 * T::RN]) {
    constexpr int BM = T::BM, BN = T::BN, RM = T::RM, RN = T::RN;
    const int tx = threadIdx.x % T::TX, ty = threadIdx.x / T::TX;
    const bool fast_c = vc && m0 + BM <= a.m && n0 + BN <= a.n;
#pragma unroll
    for (int j = 0; j < 4 * RN; ++j) {
        const int gn = n0 + (j / 4) * (BN / RN) + ty * 4 + (j & 3);
#pragma unroll
        for (int r = 0; r < RM; ++r) {
            const int gm = m0 + r * (BM / RM) + tx * 4;
            const float v0 = acc2[2 * r][j].x, v1 = acc2[2 * r][j].y, v2 = acc2[2 * r + 1][j].x,
                        v3 = acc2[2 * r + 1][j].y;
            if (fast_c) {
                store4(C + static_cast<size_t>(gn) * a.ldc + gm, make_float4(v0, v1, v2, v3), a.ep);
            } else if (gn < a.n) {
                const float vv[4] = {v0, v1, v2, v3};
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (gm + i < a.m) store_facc<OUT_F32>(C, static_cast<size_t>(gn) * a.ldc + gm + i, vv[i], a.ep);
            }
        }
    }
}

// S = 1: one CTA per tile, grid.x = M tiles. S > 1: clusters of S CTAs along x
// share a tile (grid.x = M tiles * S), CTA rank r runs K steps [r*ceil(kt/S), ...).
template <int TA, int TB, class T, int S>
__global__ void __launch_bounds__(T::THREADS, T::MINB) k_sgemm_ffma(const FfmaArgs a) {
    constexpr int BM = T::BM, BN = T::BN, BK = T::BK, RM = T::RM, RN = T::RN;
    constexpr int LDA_S = BM + (TA == 1 ? 4 : 0);   // padded when filled by transposing stores
    constexpr int LDB_S = BN + (TB == 0 ? 4 : 0);
    __shared__ __align__(16) float As[2][BK * LDA_S];
    __shared__ __align__(16) float Bs[2][BK * LDB_S];
    grid_dep_wait();
    grid_dep_launch();
    const int tid = threadIdx.x;
    const int tx = tid % T::TX, ty = tid / T::TX;
    const int rank = S > 1 ? static_cast<int>(blockIdx.x % S) : 0;
    const int m0 = static_cast<int>(blockIdx.x / S) * BM, n0 = blockIdx.y * BN;
    const bool full_m = m0 + BM <= a.m, full_n = n0 + BN <= a.n;
    const int kt_all = (a.k + BK - 1) / BK;
    const int kt_per = (kt_all + S - 1) / S;
    const int kt0 = rank * kt_per < kt_all ? rank * kt_per : kt_all;
    const int kt1 = kt0 + kt_per < kt_all ? kt0 + kt_per : kt_all;

    for (int b = blockIdx.z; b < a.batch; b += gridDim.z) {
        const float *A = a.a_arr ? a.a_arr[b] : a.A + static_cast<size_t>(b) * a.stride_a;
        const float *B = a.b_arr ? a.b_arr[b] : a.B + static_cast<size_t>(b) * a.stride_b;
        float *C = a.c_arr ? a.c_arr[b] : a.C + static_cast<size_t>(b) * a.stride_c;
        // float4 accesses need this entry's base 16-byte aligned as well
        const bool va = a.vec_a && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
        const bool vb = a.vec_b && (reinterpret_cast<uintptr_t>(B) & 15u) == 0;
        const bool vc = a.vec_c && (reinterpret_cast<uintptr_t>(C) & 15u) == 0;

        float2 acc2[2 * RM][4 * RN];  // acc2[ip][j] = outputs (rows 2ip, 2ip+1 of this thread, column j)
#pragma unroll
        for (int i = 0; i < 2 * RM; ++i)
#pragma unroll
            for (int j = 0; j < 4 * RN; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);

        float4 ra[T::CH_A], rb[T::CH_B];
        if (kt0 < kt1) {
            const int k0 = kt0 * BK;
            const bool fk = k0 + BK <= a.k;
#pragma unroll
            for (int i = 0; i < T::CH_A; ++i) load_a<TA, T>(a, A, m0, k0, tid + i * T::THREADS, va && full_m && fk, ra[i]);
#pragma unroll
            for (int i = 0; i < T::CH_B; ++i) load_b<TB, T>(a, B, n0, k0, tid + i * T::THREADS, vb && full_n && fk, rb[i]);
#pragma unroll
            for (int i = 0; i < T::CH_A; ++i) store_a<TA, T>(As[0], LDA_S, tid + i * T::THREADS, ra[i]);
#pragma unroll
            for (int i = 0; i < T::CH_B; ++i) store_b<TB, T>(Bs[0], LDB_S, tid + i * T::THREADS, rb[i]);
        }
        __syncthreads();

        for (int kt = kt0; kt < kt1; ++kt) {
            const int cur = (kt - kt0) & 1;
            const bool more = kt + 1 < kt1;
            if (more) {
                const int k0 = (kt + 1) * BK;
                const bool fk = k0 + BK <= a.k;
#pragma unroll
                for (int i = 0; i < T::CH_A; ++i)
                    load_a<TA, T>(a, A, m0, k0, tid + i * T::THREADS, va && full_m && fk, ra[i]);
#pragma unroll
                for (int i = 0; i < T::CH_B; ++i)
                    load_b<TB, T>(a, B, n0, k0, tid + i * T::THREADS, vb && full_n && fk, rb[i]);
            }
            const float *as = As[cur];
            const float *bs = Bs[cur];
            float4 fa[2][RM], fb[2][RN];
#pragma unroll
            for (int r = 0; r < RM; ++r) fa[0][r] = *reinterpret_cast<const float4 *>(&as[r * (BM / RM) + tx * 4]);
#pragma unroll
            for (int r = 0; r < RN; ++r) fb[0][r] = *reinterpret_cast<const float4 *>(&bs[r * (BN / RN) + ty * 4]);
#pragma unroll
            for (int kk = 0; kk < BK; ++kk) {
                const int f = kk & 1;
                if (kk + 1 < BK) {
#pragma unroll
                    for (int r = 0; r < RM; ++r)
                        fa[f ^ 1][r] = *reinterpret_cast<const float4 *>(&as[(kk + 1) * LDA_S + r * (BM / RM) + tx * 4]);
#pragma unroll
                    for (int r = 0; r < RN; ++r)
                        fb[f ^ 1][r] = *reinterpret_cast<const float4 *>(&bs[(kk + 1) * LDB_S + r * (BN / RN) + ty * 4]);
                }
                // Packed FP32 FMA (FFMA2): two rows of one output column per instruction, each
                // element rounded once exactly as fmaf rounds it.
#pragma unroll
                for (int j = 0; j < 4 * RN; ++j) {
                    const float4 &vb = fb[f][j / 4];
                    const float bv = (j & 3) == 0 ? vb.x : (j & 3) == 1 ? vb.y : (j & 3) == 2 ? vb.z : vb.w;
                    const float2 b2 = make_float2(bv, bv);
#pragma unroll
                    for (int ip = 0; ip < 2 * RM; ++ip) {
                        const float4 &va = fa[f][ip / 2];
                        const float2 a2 = (ip & 1) ? make_float2(va.z, va.w) : make_float2(va.x, va.y);
                        acc2[ip][j] = __ffma2_rn(a2, b2, acc2[ip][j]);
                    }
                }
            }
            if (more) {
#pragma unroll
                for (int i = 0; i < T::CH_A; ++i) store_a<TA, T>(As[cur ^ 1], LDA_S, tid + i * T::THREADS, ra[i]);
#pragma unroll
                for (int i = 0; i < T::CH_B; ++i) store_b<TB, T>(Bs[cur ^ 1], LDB_S, tid + i * T::THREADS, rb[i]);
            }
            __syncthreads();
        }

        if constexpr (S > 1) {
            // Partial tile, column-major (BM floats per column), then the cluster reduction.
            __shared__ __align__(16) float P[BM * BN];
            namespace cg = cooperative_groups;
            cg::cluster_group cluster = cg::this_cluster();
#pragma unroll
            for (int j = 0; j < 4 * RN; ++j) {
                const int ln = (j / 4) * (BN / RN) + ty * 4 + (j & 3);
#pragma unroll
                for (int r = 0; r < RM; ++r)
                    *reinterpret_cast<float4 *>(&P[ln * BM + r * (BM / RM) + tx * 4]) =
                        make_float4(acc2[2 * r][j].x, acc2[2 * r][j].y, acc2[2 * r + 1][j].x, acc2[2 * r + 1][j].y);
            }
            cluster.sync();
            const float *parts[S];
#pragma unroll
            for (int q = 0; q < S; ++q) parts[q] = cluster.map_shared_rank(P, q);
            constexpr int SLICE = BM * BN / S;   // floats of the tile this CTA finishes
            const bool fast_c = vc && full_m && full_n;
            for (int e = rank * SLICE + tid * 4; e < (rank + 1) * SLICE; e += T::THREADS * 4) {
                float4 v = *reinterpret_cast<const float4 *>(parts[0] + e);
#pragma unroll
                for (int q = 1; q < S; ++q) {
                    const float4 w = *reinterpret_cast<const float4 *>(parts[q] + e);
                    v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
                }
                const int gm = m0 + e % BM, gn = n0 + e / BM;
                if (fast_c) {
                    store4(C + static_cast<size_t>(gn) * a.ldc + gm, v, a.ep);
                } else if (gn < a.n) {
                    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (gm + i < a.m) store_facc<OUT_F32>(C, static_cast<size_t>(gn) * a.ldc + gm + i, vv[i], a.ep);
                }
            }
            cluster.sync();   // partials stay readable until every CTA of the cluster is done
        } else {
        float acc[4 * RM][4 * RN];
#pragma unroll
        for (int i = 0; i < 2 * RM; ++i)
#pragma unroll
            for (int j = 0; j < 4 * RN; ++j) {
                acc[2 * i][j] = acc2[i][j].x;
                acc[2 * i + 1][j] = acc2[i][j].y;
            }
        // Epilogue: rows m0 + r*(BM/RM) + tx*4 + {0..3}, columns n0 + s*(BN/RN) + ty*4 + {0..3}.
        // alpha*acc then + beta*C with separate roundings, as gemm(f32) does (src/gemm.zig:523-544).
        const bool fast_c = vc && full_m && full_n;
#pragma unroll
        for (int j = 0; j < 4 * RN; ++j) {
            const int gn = n0 + (j / 4) * (BN / RN) + ty * 4 + (j & 3);
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                const int gm = m0 + r * (BM / RM) + tx * 4;
                float *p = C + static_cast<size_t>(gn) * a.ldc + gm;
                if (fast_c) {
                    store4(p, make_float4(acc[r * 4 + 0][j], acc[r * 4 + 1][j], acc[r * 4 + 2][j], acc[r * 4 + 3][j]),
                           a.ep);
                } else if (gn < a.n) {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (gm + i < a.m) store_facc<OUT_F32>(C, static_cast<size_t>(gn) * a.ldc + gm + i, acc[r * 4 + i][j], a.ep);
                }
            }
        }
        }
    }
}

// ---- stream-K: the (tile, K step) iterations of a launch spread evenly over the CTAs -------------------
//
// A launch of TileL tiles leaves SMs idle when its tile count is not a multiple of the 2 x 148 resident
// CTAs (C2's 4096 x 1024 has 256 tiles: 40 SMs hold one CTA, 108 hold two, 13.5 % of the slots empty). The
// stream-K kernel launches exactly the resident CTAs and gives CTA c the iterations [c*T/G, (c+1)*T/G)
// of the T = tiles x K-steps iterations, tile by tile in order. A tile covered by one CTA is stored
// directly. A tile split between CTAs is finished by the last of them to arrive: every contributor writes
// its partial tile to its own workspace slot (one for the first tile of its range, one for the last), then
// adds its K-step count to the tile's counter; the CTA whose addition completes the count sums all
// contributors' slots in K order (the same order whoever arrives last, so results are deterministic),
// applies alpha / beta, stores the tile and resets the counter for the next launch. No CTA waits for
// another, so nothing depends on the CTAs being co-resident.

struct SkArgs {
    long long tiles;      // m tiles x n tiles x batch
    int mt, nt;           // tile counts along M and N
    int kt;               // K steps per tile
    float4 *partials;     // 2 slots of BM x BN floats per CTA
    unsigned *counts;     // per tile: K steps accumulated by partial contributors so far (0 between launches)
};

__device__ __forceinline__ long long sk_begin(long long c, long long total, long long g) { return c * total / g; }

// The CTA whose iteration range holds iteration i.
__device__ __forceinline__ long long sk_owner(long long i, long long total, long long g) {
    long long c = i * g / total;
    while (c + 1 < g && sk_begin(c + 1, total, g) <= i) ++c;
    while (c > 0 && sk_begin(c, total, g) > i) --c;
    return c;
}

template <int TA, int TB, class T>
__global__ void __launch_bounds__(T::THREADS, T::MINB) k_sgemm_ffma_sk(const FfmaArgs a, const SkArgs s) {
    constexpr int BM = T::BM, BN = T::BN, RM = T::RM, RN = T::RN;
    constexpr int Q = BM * BN / 4 / T::THREADS;  // float4 of a partial tile per thread
    static_assert(Q * 4 == 2 * RM * 4 * RN * 2, "partial tile / accumulator mismatch");
    __shared__ __align__(16) float As[2][T::BK * Smem<TA, TB, T>::LDA_S];
    __shared__ __align__(16) float Bs[2][T::BK * Smem<TA, TB, T>::LDB_S];
    __shared__ int is_last;
    grid_dep_wait();
    grid_dep_launch();
    const int tid = threadIdx.x;
    const long long g = gridDim.x, c = blockIdx.x;
    const long long total = s.tiles * s.kt;
    const long long beg = sk_begin(c, total, g), end = sk_begin(c + 1, total, g);
    const long long first_tile = beg / s.kt;
    for (long long it = beg; it < end;) {
        const long long tile = it / s.kt;
        const int kb = static_cast<int>(it - tile * s.kt);
        const int ke = static_cast<int>(end - tile * s.kt < s.kt ? end - tile * s.kt : s.kt);
        const long long per_batch = static_cast<long long>(s.mt) * s.nt;
        const int b = static_cast<int>(tile / per_batch);
        const int r = static_cast<int>(tile - b * per_batch);
        const int m0 = (r % s.mt) * BM, n0 = (r / s.mt) * BN;
        const float *A = a.A + static_cast<size_t>(b) * a.stride_a;
        const float *B = a.B + static_cast<size_t>(b) * a.stride_b;
        float *C = a.C + static_cast<size_t>(b) * a.stride_c;
        const bool va = a.vec_a && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
        const bool vb = a.vec_b && (reinterpret_cast<uintptr_t>(B) & 15u) == 0;
        const bool vc = a.vec_c && (reinterpret_cast<uintptr_t>(C) & 15u) == 0;

        float2 acc2[2 * RM][4 * RN];
#pragma unroll
        for (int i = 0; i < 2 * RM; ++i)
#pragma unroll
            for (int j = 0; j < 4 * RN; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
        k_loop<TA, TB, T>(a, A, B, m0, n0, kb, ke, va, vb, As, Bs, acc2);

        if (kb == 0 && ke == s.kt) {
            store_tile<T>(a, C, m0, n0, vc, acc2);
        } else {
            // Partial tile: this CTA's slot for it, float4 q of thread tid at q * THREADS + tid.
            float4 *slot = s.partials + (2 * c + (tile == first_tile ? 0 : 1)) * (BM * BN / 4);
#pragma unroll
            for (int q = 0; q < Q; ++q) {
                const int ip = (2 * q) / (4 * RN), j = (2 * q) % (4 * RN);
                slot[q * T::THREADS + tid] = make_float4(acc2[ip][j].x, acc2[ip][j].y, acc2[ip][j + 1].x,
                                                         acc2[ip][j + 1].y);
            }
            __threadfence();
            __syncthreads();
            if (tid == 0) {
                const unsigned add = static_cast<unsigned>(ke - kb);
                is_last = atomicAdd(&s.counts[tile], add) + add == static_cast<unsigned>(s.kt);
            }
            __syncthreads();
            if (is_last) {
                __threadfence();
                // Sum the contributors' slots in K order (the CTAs whose ranges meet this tile).
                const long long t0 = tile * s.kt;
                const long long c_lo = sk_owner(t0, total, g), c_hi = sk_owner(t0 + s.kt - 1, total, g);
#pragma unroll
                for (int i = 0; i < 2 * RM; ++i)
#pragma unroll
                    for (int j = 0; j < 4 * RN; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
                for (long long cc = c_lo; cc <= c_hi; ++cc) {
                    const long long cc_first = sk_begin(cc, total, g) / s.kt;
                    const float4 *src = s.partials + (2 * cc + (tile == cc_first ? 0 : 1)) * (BM * BN / 4);
#pragma unroll
                    for (int q = 0; q < Q; ++q) {
                        const int ip = (2 * q) / (4 * RN), j = (2 * q) % (4 * RN);
                        const float4 v = __ldcg(src + q * T::THREADS + tid);
                        acc2[ip][j].x += v.x;
                        acc2[ip][j].y += v.y;
                        acc2[ip][j + 1].x += v.z;
                        acc2[ip][j + 1].y += v.w;
                    }
                }
                store_tile<T>(a, C, m0, n0, vc, acc2);
                if (tid == 0) s.counts[tile] = 0;  // ready for the next launch
            }
        }
        it = tile * s.kt + ke;
    }
}

template <int TA, int TB, class T, int S>
static cudaError_t go(Context &ctx, const FfmaArgs &a) {
    dim3 grid((a.m + T::BM - 1) / T::BM * S, (a.n + T::BN - 1) / T::BN, a.batch < 65535 ? a.batch : 65535);
    const cudaError_t e = launch_pdl(k_sgemm_ffma<TA, TB, T, S>, grid, dim3(T::THREADS), 0, ctx.stream, S, a);
    ctx.launches++;
    return e;
}

template <class T, int S = 1>
static cudaError_t go_ops(Context &ctx, const GemmDesc &d, const FfmaArgs &a) {
    if (!d.trans_a && !d.trans_b) return go<0, 0, T, S>(ctx, a);
    if (!d.trans_a && d.trans_b) return go<0, 1, T, S>(ctx, a);
    if (d.trans_a && !d.trans_b) return go<1, 0, T, S>(ctx, a);
    return go<1, 1, T, S>(ctx, a);
}

template <class T>
static long long ctas(const GemmDesc &d) {
    return static_cast<long long>((d.m + T::BM - 1) / T::BM) * ((d.n + T::BN - 1) / T::BN) * d.batch;
}

// Stream-K launch over exactly the resident CTAs of tile T. The workspace (two partial tiles per CTA) and
// the per-tile counters are handle-owned, separate and grow-only; counters are zeroed when allocated and
// reset by the kernel after use, so every launch finds them at zero.
template <int TA, int TB, class T>
static cudaError_t go_sk(Context &ctx, const FfmaArgs &a, long long ctas_resident) {
    SkArgs s{};
    s.mt = (a.m + T::BM - 1) / T::BM;
    s.nt = (a.n + T::BN - 1) / T::BN;
    s.tiles = static_cast<long long>(s.mt) * s.nt * a.batch;
    s.kt = (a.k + T::BK - 1) / T::BK;
    const long long grid = ctas_resident;
    const size_t part_bytes = static_cast<size_t>(grid) * 2 * T::BM * T::BN * sizeof(float);
    const size_t count_bytes = static_cast<size_t>(s.tiles) * sizeof(unsigned);
    if (ctx.sk_bytes < part_bytes || ctx.sk_count_bytes < count_bytes) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(ctx.stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
            ctx.last_error = "the FP32 stream-K workspace must grow, which cannot be captured: make one call of "
                             "this size before the stream capture";
            return cudaErrorStreamCaptureUnsupported;
        }
    }
    if (ctx.sk_bytes < part_bytes) {
        const size_t bytes = part_bytes > 2 * ctx.sk_bytes ? part_bytes : 2 * ctx.sk_bytes;
        void *grown = nullptr;
        const cudaError_t e = cudaMalloc(&grown, bytes);
        if (e != cudaSuccess) return e;
        if (ctx.sk_buf) ctx.retired.push_back(ctx.sk_buf);  // kernels in flight may still read it
        ctx.sk_buf = grown;
        ctx.sk_bytes = bytes;
    }
    if (ctx.sk_count_bytes < count_bytes) {
        const size_t bytes = count_bytes > 2 * ctx.sk_count_bytes ? count_bytes : 2 * ctx.sk_count_bytes;
        void *grown = nullptr;
        cudaError_t e = cudaMalloc(&grown, bytes);
        if (e != cudaSuccess) return e;
        e = cudaMemsetAsync(grown, 0, bytes, ctx.stream);  // counters start at zero; kernels leave them zero
        if (e != cudaSuccess) {
            cudaFree(grown);
            return e;
        }
        if (ctx.sk_counts) ctx.retired.push_back(ctx.sk_counts);
        ctx.sk_counts = grown;
        ctx.sk_count_bytes = bytes;
    }
    s.partials = static_cast<float4 *>(ctx.sk_buf);
    s.counts = static_cast<unsigned *>(ctx.sk_counts);
    const cudaError_t e = launch_pdl(k_sgemm_ffma_sk<TA, TB, T>, dim3(static_cast<unsigned>(grid)), dim3(T::THREADS),
                                     0, ctx.stream, 1, a, s);
    ctx.launches++;
    return e;
}

// Share of the resident CTA slots a data-parallel launch of `tiles` tiles keeps busy over its waves.
static double wave_use(long long tiles, long long slots) {
    const long long waves = (tiles + slots - 1) / slots;
    return static_cast<double>(tiles) / static_cast<double>(waves * slots);
}

}  // namespace ffma

// Tile choice: the largest tile whose grid still gives every SM at least one
// CTA; below that the 64 x 64 tile with K split over a cluster of S CTAs
// (S the power of two, at most 8, that brings the grid to the SM count while
// every CTA keeps at least two K steps, doubled once more for grids of at
// most half the SM count); the 32 x 32 tile when K is too short to split.
// a_arr/b_arr/c_arr: device arrays of per-entry pointers (pointer-array
// batches), or nullptr for the strided layout of `d`.
cudaError_t launch_ffma_ptr(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                            void *const *c_arr) {
    using namespace ffma;
    // Column tiles are grid.y (at most 65535 blocks): wider problems run as
    // column slices that every tile size can cover (B and C offset per slice).
    constexpr long long kSliceCols = 65535LL * 32;
    if (d.n > kSliceCols) {
        if (a_arr != nullptr) return cudaErrorInvalidValue;  // per-entry pointers cannot be offset here
        for (long long j0 = 0; j0 < d.n; j0 += kSliceCols) {
            GemmDesc s = d;
            s.n = static_cast<int>(d.n - j0 < kSliceCols ? d.n - j0 : kSliceCols);
            s.B = static_cast<const float *>(d.B) + (d.trans_b ? j0 : j0 * d.ldb);
            s.C = static_cast<float *>(d.C) + j0 * d.ldc;
            const cudaError_t e = launch_ffma_ptr(ctx, s, nullptr, nullptr, nullptr);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    FfmaArgs a{};
    a.a_arr = reinterpret_cast<const float *const *>(a_arr);
    a.b_arr = reinterpret_cast<const float *const *>(b_arr);
    a.c_arr = reinterpret_cast<float *const *>(c_arr);
    a.m = d.m;
    a.n = d.n;
    a.k = d.k;
    a.batch = d.batch;
    a.A = static_cast<const float *>(d.A); a.lda = d.lda; a.stride_a = d.stride_a;
    a.B = static_cast<const float *>(d.B); a.ldb = d.ldb; a.stride_b = d.stride_b;
    a.C = static_cast<float *>(d.C); a.ldc = d.ldc; a.stride_c = d.stride_c;
    const bool strided = d.batch > 1 && a_arr == nullptr;
    a.vec_a = d.lda % 4 == 0 && (!strided || d.stride_a % 4 == 0);
    a.vec_b = d.ldb % 4 == 0 && (!strided || d.stride_b % 4 == 0);
    a.vec_c = d.ldc % 4 == 0 && (!strided || d.stride_c % 4 == 0);
    a.ep = d.ep;
    const long long sms = ctx.sm_count > 0 ? ctx.sm_count : 148;
    const long long cm = ctas<TileM>(d);
    // op(A) = T with op(B) = N is the one 128 x 128 variant that spills at 128
    // registers; the 64 x 64 tile is faster for it whenever its grid fills the GPU.
    const bool tn = d.trans_a && !d.trans_b;
    // Stream-K for a single partial wave of 128 x 128 tiles (at least one per SM, fewer than two full
    // waves, more than a tenth of the resident slots idle) whose tiles have at least 64 K steps to amortise
    // the partial-tile exchange: C2's 4096 x 1024 x 2048 (256 tiles on 296 slots) and 2048^3 measured 5-6 %
    // faster. Measured slower and kept data-parallel: 32 K steps (1024 x 4096 x 512, 9 %), several waves
    // (4096^3, 6 % even with the leading waves run data-parallel), and op T/N on the 64 x 64 tile (4-5 %).
    // Handle calls only: it needs a workspace; pointer-array batches keep the per-entry grid.
    const long long ctas_l = ctas<TileL>(d), slots = 2 * sms;
    const int kt_l = (d.k + TileL::BK - 1) / TileL::BK;
    if (ctx.may_allocate && a_arr == nullptr && !tn && ctas_l >= sms && ctas_l < 2 * slots && kt_l >= 64 &&
        wave_use(ctas_l, slots) < 0.9) {
        const cudaError_t e = !d.trans_a && !d.trans_b ? go_sk<0, 0, TileL>(ctx, a, slots)
                              : !d.trans_a            ? go_sk<0, 1, TileL>(ctx, a, slots)
                                                      : go_sk<1, 1, TileL>(ctx, a, slots);
        if (e != cudaErrorMemoryAllocation) return e;
        cudaGetLastError();  // no room for the workspace: the data-parallel grid below needs none
    }
    if (ctas_l >= sms && !(tn && cm >= sms)) return go_ops<TileL>(ctx, d, a);
    if (cm >= sms) return go_ops<TileM>(ctx, d, a);
    const int ksteps = (d.k + TileM::BK - 1) / TileM::BK;
    int split = 1;
    while (split < 8 && cm * split < sms && ksteps >= 4 * split) split *= 2;
    // At most half the SMs' worth of tiles: one more doubling measured faster (512^3: 4 -> 8).
    if (split > 1 && split < 8 && 2 * cm <= sms && ksteps >= 8 * split) split *= 2;
    if (split == 8) return go_ops<TileM, 8>(ctx, d, a);
    if (split == 4) return go_ops<TileM, 4>(ctx, d, a);
    if (split == 2) return go_ops<TileM, 2>(ctx, d, a);
    return go_ops<TileS>(ctx, d, a);
}

cudaError_t launch_ffma(Context &ctx, const GemmDesc &d) { return launch_ffma_ptr(ctx, d, nullptr, nullptr, nullptr); }

}  // namespace gs
