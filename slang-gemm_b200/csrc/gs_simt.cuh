// gs_simt.cuh -- the CUDA-core GEMM tile loop, shared by the stand-alone
// CUDA-core kernel (gemm_simt.cu) and the tensor-core kernel's fallback for
// pointer-array batches whose pointers TMA cannot address.
//
// B200 counterpart of slang-gemm's generic fallback shaders
// (shaders/gemm_lowp_f32.slang, shaders/gemm_integer_i32.slang): any op, any
// stride, f16/bf16/f32 inputs with f32 accumulation, s8 inputs with s32
// accumulation, 64 x 64 output tiles computed by 256 threads.
#pragma once
#include <type_traits>

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
    Epilogue ep;
};

template <int IN>
__device__ __forceinline__ auto load_elem(const void *p, size_t i) {
    if constexpr (IN == IN_F16) return __half2float(static_cast<const __half *>(p)[i]);
    else if constexpr (IN == IN_BF16) return bf16_bits_to_f32(static_cast<const uint16_t *>(p)[i]);
    else if constexpr (IN == IN_F32) return static_cast<const float *>(p)[i];
    else return static_cast<int32_t>(static_cast<const int8_t *>(p)[i]);
}

// Arguments of the tile loop for a validated problem; a_arr/b_arr/c_arr are
// device arrays of per-entry pointers (pointer-array batches) or nullptr.
inline SimtArgs make_args(const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                          void *const *c_arr) {
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
    s.ep = d.ep;
    return s;
}

// Shared memory the tile loop needs (A and B panels of one K step).
template <int IN>
constexpr size_t tile_smem_bytes() {
    using Acc = typename std::conditional<IN == IN_I8, int32_t, float>::type;
    return sizeof(Acc) * (TK * TM + TK * (TN + 1));
}

// Computes the 64 x 64 output tiles first, first + step, ... of every batch
// entry (tiles numbered M-block fastest, then N-block, then batch entry).
// Threads 0..255 of the block do the work; every thread of the block must
// call this function (it synchronises the block).
template <int IN, int OUT>
__device__ __forceinline__ void simt_tiles(const SimtArgs &a, long long first, long long step, void *smem) {
    using Acc = typename std::conditional<IN == IN_I8, int32_t, float>::type;
    Acc (*As)[TM] = reinterpret_cast<Acc (*)[TM]>(smem);
    Acc (*Bs)[TN + 1] = reinterpret_cast<Acc (*)[TN + 1]>(static_cast<Acc *>(smem) + TK * TM);
    const int tid = threadIdx.x;
    const bool worker = tid < 256;
    const int tx = tid & 15, ty = (tid >> 4) & 15;
    const long long mt = (a.m + TM - 1) / TM, nt = (a.n + TN - 1) / TN;
    const long long total = mt * nt * a.batch;
    for (long long t = first; t < total; t += step) {
        const int b = static_cast<int>(t / (mt * nt));
        const long long r = t - static_cast<long long>(b) * mt * nt;
        const int m0 = static_cast<int>(r % mt) * TM, n0 = static_cast<int>(r / mt) * TN;
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
            if (worker) {
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
            }
            __syncthreads();
            if (worker) {
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
            }
            __syncthreads();
        }
        if (worker) {
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
}

}  // namespace simt
}  // namespace gs
