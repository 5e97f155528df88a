// gemm_tc_sm100.cu -- tcgen05 tensor-core GEMM for sm_100a.
//
// Computes C = alpha * op(A) * op(B) + beta * C, column-major, for
//   f16 x f16 -> f32 / f16 and bf16 x bf16 -> f32 / bf16  (tcgen05.mma kind::f16)
//   s8 x s8 -> s32                                         (tcgen05.mma kind::i8)
// It replaces slang-gemm's cooperative-matrix shaders
// (shaders/gemm_nvcoop2_f16.slang, shaders/gemm_nvcoop2_i8.slang and the bf16
// path of tools/emit_nvcoop2_spv.zig); the arithmetic contract is gemmExCuda
// (src/gemm.zig:671-706).
//
// Design (one CTA per SM, persistent over output tiles):
//  - tile 128 (M) x 256 (N), 128 bytes of K per pipeline stage, 4 stages;
//  - warp 0: TMA producer. Operand transposes live in the tensor maps: op(A)=N
//    (M-contiguous) and op(B)=T (N-contiguous) are fetched as MN-major 128-byte
//    swizzled panels, op(A)=T and op(B)=N as K-major panels, and the UMMA
//    instruction descriptor's major bits tell the tensor core which is which;
//  - warp 1: allocates 512 TMEM columns (two 128x256 accumulators) and issues
//    tcgen05.mma from one thread; tcgen05.commit frees smem stages and
//    publishes finished accumulators;
//  - warps 2..5: epilogue. tcgen05.ld pulls one accumulator row per thread;
//    because C is column-major, the 32 lanes of a warp store 32 consecutive
//    rows of one column (one 128-byte segment per instruction for f32/i32).
//    Double-buffered TMEM lets the epilogue of tile i overlap the main loop of
//    tile i+1.
// Batches (strided or pointer-array) are the outermost tile coordinate; the
// M/N tiles of one batch are visited in groups of `group_m` row blocks so
// that concurrently running CTAs share A and B panels in L2.
#include <cstdio>

#include "gs_epilogue.cuh"
#include "gs_internal.h"
#include "gs_ptx.cuh"

namespace gs {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK_BYTES = 128;
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK_BYTES;  // 16 KiB
constexpr int B_STAGE_BYTES = BN * BK_BYTES;  // 32 KiB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*alignment slack*/ + 256 /*barriers*/;

struct TcArgs {
    int m, n, k, batch;
    int m_blocks, n_blocks, k_blocks;
    long long tiles_per_batch, total_tiles;
    int a_mn, b_mn;        // operand stored MN-major (A op N, B op T)
    int a_bcast, b_bcast;  // batch coordinate pinned to 0 (stride 0)
    int group_m;
    void *C;
    long long ldc, stride_c;
    void *const *c_arr;          // pointer-array batches: per-batch C
    const CUtensorMap *a_maps;   // pointer-array batches: per-batch maps in global memory
    const CUtensorMap *b_maps;
    const uint32_t *skip_flag;   // pointer-array batches: set when a pointer is not 16-byte aligned
    Epilogue ep;
    uint32_t *err;
};

__device__ __forceinline__ void tile_coords(const TcArgs &a, long long t, int &b, int &mb, int &nb) {
    b = static_cast<int>(t / a.tiles_per_batch);
    const long long r = t - static_cast<long long>(b) * a.tiles_per_batch;
    const long long span = static_cast<long long>(a.group_m) * a.n_blocks;
    const int g = static_cast<int>(r / span);
    const int within = static_cast<int>(r - g * span);
    const int first_m = g * a.group_m;
    const int gm = min(a.group_m, a.m_blocks - first_m);
    mb = first_m + within % gm;
    nb = within / gm;
}

template <int IN, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcArgs args) {
    constexpr int ES = (IN == IN_I8) ? 1 : 2;          // element bytes
    constexpr int BK = BK_BYTES / ES;                  // K elements per stage
    constexpr int UK = (IN == IN_I8) ? 32 : 16;        // K per tcgen05.mma
    constexpr int CH = BK_BYTES / ES;                  // MN elements per 128-byte swizzle panel
    constexpr uint32_t CH_BYTES = CH * BK * ES;        // bytes of one MN-major panel (BK rows x 128 B)
    constexpr uint32_t C_FMT = (IN == IN_I8) ? 2u : 1u;
    constexpr uint32_t AB_FMT = (IN == IN_F16) ? 0u : 1u;  // bf16 = 1, s8 = 1

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *smA = smem;
    uint8_t *smB = smem + STAGES * A_STAGE_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smB + STAGES * B_STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Pointer-array batches whose pointers TMA cannot address are computed by
    // the CUDA-core kernel launched after this one instead.
    if (args.skip_flag != nullptr && *args.skip_flag != 0u) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 128);
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0 && args.a_maps == nullptr) {
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (long long t = blockIdx.x; ok && t < args.total_tiles; t += gridDim.x) {
                int b, mb, nb;
                tile_coords(args, t, b, mb, nb);
                const int m0 = mb * BM, n0 = nb * BN;
                const CUtensorMap *ma = &tmA, *mbp = &tmB;
                int ab = args.a_bcast ? 0 : b, bb = args.b_bcast ? 0 : b;
                if (args.a_maps != nullptr) {
                    ma = args.a_maps + b;
                    mbp = args.b_maps + b;
                    ab = 0;
                    bb = 0;
                    tensormap_acquire(ma);
                    tensormap_acquire(mbp);
                }
                for (int kb = 0; kb < args.k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, 1)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    uint8_t *dA = smA + stage * A_STAGE_BYTES;
                    uint8_t *dB = smB + stage * B_STAGE_BYTES;
                    const int k0 = kb * BK;
                    if (args.a_mn) {
#pragma unroll
                        for (int c = 0; c < BM / CH; ++c) tma_load_3d(dA + c * CH_BYTES, ma, &full[stage], m0 + c * CH, k0, ab);
                    } else {
                        tma_load_3d(dA, ma, &full[stage], k0, m0, ab);
                    }
                    if (args.b_mn) {
#pragma unroll
                        for (int c = 0; c < BN / CH; ++c) tma_load_3d(dB + c * CH_BYTES, mbp, &full[stage], n0 + c * CH, k0, bb);
                    } else {
                        tma_load_3d(dB, mbp, &full[stage], k0, n0, bb);
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(C_FMT, AB_FMT, args.a_mn, args.b_mn, BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (long long t = blockIdx.x; ok && t < args.total_tiles; t += gridDim.x, ++it) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.err, 2)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < args.k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, args.err, 3)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(smA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(smB + stage * B_STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UK; ++kk) {
                        const uint64_t adesc = args.a_mn ? umma_smem_desc_sw128(a_base + kk * UK * 128, CH_BYTES, 1024)
                                                         : umma_smem_desc_sw128(a_base + kk * UK * ES, 16, 1024);
                        const uint64_t bdesc = args.b_mn ? umma_smem_desc_sw128(b_base + kk * UK * 128, CH_BYTES, 1024)
                                                         : umma_smem_desc_sw128(b_base + kk * UK * ES, 16, 1024);
                        if constexpr (IN == IN_I8) umma_i8(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0);
                        else umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (ok) umma_commit(&tfull[acc]);
            }
        }
    } else {
        // ---------------- epilogue warps 2..5 ----------------
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        int it = 0;
        for (long long t = blockIdx.x; t < args.total_tiles; t += gridDim.x, ++it) {
            int b, mb, nb;
            tile_coords(args, t, b, mb, nb);
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, args.err, 4)) break;
            tc_fence_after();
            const int m = mb * BM + row;
            const int n0 = nb * BN;
            void *Cb = args.C;
            if (args.c_arr != nullptr) Cb = args.c_arr[b];
            else Cb = static_cast<uint8_t *>(args.C) + static_cast<size_t>(b) * args.stride_c *
                                                        ((OUT == OUT_F16 || OUT == OUT_BF16) ? 2 : 4);
            const int ncols = min(BN, args.n - n0);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN + c, r);
                tmem_wait_ld();
                if (m < args.m && c < ncols) {
                    const int jn = min(32, ncols - c);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (j < jn) {
                            const size_t idx = static_cast<size_t>(m) + static_cast<size_t>(n0 + c + j) * args.ldc;
                            if constexpr (OUT == OUT_I32) store_iacc(Cb, idx, static_cast<int32_t>(r[j]), args.ep);
                            else store_facc<OUT>(Cb, idx, __uint_as_float(r[j]), args.ep);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Kernel that writes one tensor map per pointer-array batch entry: it copies
// a host-encoded template and patches the global address with
// tensormap.replace, then makes the write visible to the tensor-map proxy.
// A pointer that is not 16-byte aligned cannot be a TMA base address: the
// builder then raises *misaligned, the tensor-core kernel returns at once and
// the CUDA-core kernel computes the whole batch instead.
__global__ void k_build_ptr_maps(const CUtensorMap tmpl_a, const CUtensorMap tmpl_b, const void *const *a_arr,
                                 const void *const *b_arr, CUtensorMap *maps_a, CUtensorMap *maps_b, int batch,
                                 uint32_t *misaligned) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch) return;
    const uint64_t pa = reinterpret_cast<uint64_t>(a_arr[i]), pb = reinterpret_cast<uint64_t>(b_arr[i]);
    if (((pa | pb) & 15u) != 0u) {
        atomicOr(misaligned, 1u);
        return;
    }
    maps_a[i] = tmpl_a;
    maps_b[i] = tmpl_b;
    asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;"
                 ::"l"(reinterpret_cast<uint64_t>(maps_a + i)), "l"(reinterpret_cast<uint64_t>(a_arr[i])) : "memory");
    asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;"
                 ::"l"(reinterpret_cast<uint64_t>(maps_b + i)), "l"(reinterpret_cast<uint64_t>(b_arr[i])) : "memory");
    asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
}

template <int IN, int OUT>
static cudaError_t launch_kernel(Context &ctx, const CUtensorMap &ta, const CUtensorMap &tb, const TcArgs &args) {
    auto kern = k_gemm_tc<IN, OUT>;
    static bool attr_set[64] = {};  // per instantiation and device
    cudaError_t e = cudaSuccess;
    if (ctx.device < 0 || ctx.device >= 64 || !attr_set[ctx.device]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (ctx.device >= 0 && ctx.device < 64) attr_set[ctx.device] = true;
    }
    const long long grid = args.total_tiles < ctx.sm_count ? args.total_tiles : ctx.sm_count;
    kern<<<static_cast<unsigned>(grid), NUM_THREADS, SMEM_BYTES, ctx.stream>>>(ta, tb, args);
    ctx.launches++;
    return cudaGetLastError();
}

static cudaError_t dispatch(Context &ctx, const GemmDesc &d, const CUtensorMap &ta, const CUtensorMap &tb,
                            const TcArgs &args) {
    switch (d.in_kind) {
    case IN_F16:
        if (d.out_kind == OUT_F32) return launch_kernel<IN_F16, OUT_F32>(ctx, ta, tb, args);
        if (d.out_kind == OUT_F16) return launch_kernel<IN_F16, OUT_F16>(ctx, ta, tb, args);
        break;
    case IN_BF16:
        if (d.out_kind == OUT_F32) return launch_kernel<IN_BF16, OUT_F32>(ctx, ta, tb, args);
        if (d.out_kind == OUT_BF16) return launch_kernel<IN_BF16, OUT_BF16>(ctx, ta, tb, args);
        break;
    case IN_I8:
        if (d.out_kind == OUT_I32) return launch_kernel<IN_I8, OUT_I32>(ctx, ta, tb, args);
        break;
    default: break;
    }
    return cudaErrorInvalidValue;
}

static CUtensorMapDataType tmap_dtype(InKind k) {
    return k == IN_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                       : (k == IN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8);
}

// Encodes the A and B maps. `batch_a`/`batch_b` are the extents of the third
// (batch) dimension: 1 when every batch entry reads the same matrix.
static bool make_maps(const GemmDesc &d, const void *a_base, const void *b_base, int batch_a, int batch_b,
                      CUtensorMap *ta, CUtensorMap *tb, std::string *why) {
    const size_t es = in_elem_size(d.in_kind);
    const uint32_t bk = BK_BYTES / static_cast<uint32_t>(es);
    const uint32_t ch = BK_BYTES / static_cast<uint32_t>(es);
    const CUtensorMapDataType dt = tmap_dtype(d.in_kind);
    // A: op N -> stored m x k (M-contiguous); op T -> stored k x m (K-contiguous).
    const uint64_t a0 = d.trans_a ? d.k : d.m, a1 = d.trans_a ? d.m : d.k;
    const uint64_t a_s1 = static_cast<uint64_t>(d.lda) * es;
    const uint64_t a_s2 = batch_a > 1 ? static_cast<uint64_t>(d.stride_a) * es : a1 * a_s1;
    if (!encode_tmap_3d(ta, dt, a_base, a0, a1, static_cast<uint64_t>(batch_a), a_s1, a_s2,
                        d.trans_a ? bk : ch, d.trans_a ? static_cast<uint32_t>(BM) : bk, why))
        return false;
    // B: op N -> stored k x n (K-contiguous); op T -> stored n x k (N-contiguous).
    const uint64_t b0 = d.trans_b ? d.n : d.k, b1 = d.trans_b ? d.k : d.n;
    const uint64_t b_s1 = static_cast<uint64_t>(d.ldb) * es;
    const uint64_t b_s2 = batch_b > 1 ? static_cast<uint64_t>(d.stride_b) * es : b1 * b_s1;
    if (!encode_tmap_3d(tb, dt, b_base, b0, b1, static_cast<uint64_t>(batch_b), b_s1, b_s2,
                        d.trans_b ? ch : bk, d.trans_b ? bk : static_cast<uint32_t>(BN), why))
        return false;
    return true;
}

static TcArgs make_args(Context &ctx, const GemmDesc &d) {
    const int es = static_cast<int>(in_elem_size(d.in_kind));
    const int bk = BK_BYTES / es;
    TcArgs a{};
    a.m = d.m;
    a.n = d.n;
    a.k = d.k;
    a.batch = d.batch;
    a.m_blocks = (d.m + BM - 1) / BM;
    a.n_blocks = (d.n + BN - 1) / BN;
    a.k_blocks = (d.k + bk - 1) / bk;
    a.tiles_per_batch = static_cast<long long>(a.m_blocks) * a.n_blocks;
    a.total_tiles = a.tiles_per_batch * d.batch;
    a.a_mn = d.trans_a ? 0 : 1;
    a.b_mn = d.trans_b ? 1 : 0;
    a.a_bcast = (d.batch == 1 || d.stride_a == 0) ? 1 : 0;
    a.b_bcast = (d.batch == 1 || d.stride_b == 0) ? 1 : 0;
    a.group_m = a.m_blocks < 16 ? a.m_blocks : 16;
    a.C = d.C;
    a.ldc = d.ldc;
    a.stride_c = d.stride_c;
    a.c_arr = nullptr;
    a.a_maps = nullptr;
    a.b_maps = nullptr;
    a.skip_flag = nullptr;
    a.ep = d.ep;
    a.err = ctx.dev_err;
    return a;
}

}  // namespace tc

cudaError_t launch_tc(Context &ctx, const GemmDesc &d) {
    using namespace tc;
    TcArgs args = make_args(ctx, d);
    CUtensorMap ta, tb;
    std::string why;
    if (!make_maps(d, d.A, d.B, args.a_bcast ? 1 : d.batch, args.b_bcast ? 1 : d.batch, &ta, &tb, &why)) {
        ctx.last_error = "tensor map encode failed: " + why;
        return cudaErrorInvalidValue;
    }
    return dispatch(ctx, d, ta, tb, args);
}

cudaError_t launch_tc_ptr_array(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                                void *const *c_arr) {
    using namespace tc;
    TcArgs args = make_args(ctx, d);
    // Template maps over a placeholder (16-byte aligned, never dereferenced
    // through the template) with the per-batch geometry; the builder kernel
    // swaps in each batch entry's address.
    const size_t need = 2 * static_cast<size_t>(d.batch) * sizeof(CUtensorMap);
    if (ctx.tmap_bytes < need) {
        if (ctx.tmap_buf) cudaFree(ctx.tmap_buf);
        ctx.tmap_buf = nullptr;
        ctx.tmap_bytes = 0;
        cudaError_t e = cudaMalloc(&ctx.tmap_buf, need);
        if (e != cudaSuccess) return e;
        ctx.tmap_bytes = need;
    }
    CUtensorMap ta, tb;
    std::string why;
    const void *placeholder = ctx.tmap_buf;
    if (!make_maps(d, placeholder, placeholder, 1, 1, &ta, &tb, &why)) {
        ctx.last_error = "tensor map encode failed: " + why;
        return cudaErrorInvalidValue;
    }
    CUtensorMap *maps_a = static_cast<CUtensorMap *>(ctx.tmap_buf);
    CUtensorMap *maps_b = maps_a + d.batch;
    uint32_t *misaligned = ctx.dev_err + 1;
    cudaError_t e0 = cudaMemsetAsync(misaligned, 0, sizeof(uint32_t), ctx.stream);
    if (e0 != cudaSuccess) return e0;
    const int threads = 128;
    k_build_ptr_maps<<<(d.batch + threads - 1) / threads, threads, 0, ctx.stream>>>(ta, tb, a_arr, b_arr, maps_a,
                                                                                     maps_b, d.batch, misaligned);
    ctx.launches++;
    ctx.last_kernels |= GS_KERNEL_TMAP;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    args.a_bcast = 1;
    args.b_bcast = 1;
    args.a_maps = maps_a;
    args.b_maps = maps_b;
    args.c_arr = c_arr;
    args.skip_flag = misaligned;
    e = dispatch(ctx, d, ta, tb, args);
    if (e != cudaSuccess) return e;
    // Runs only when the builder raised the flag (it reads the same word).
    return launch_simt_if_flag(ctx, d, a_arr, b_arr, c_arr, misaligned);
}

}  // namespace gs
