// gemm_tc_sm100.cu -- tcgen05 tensor-core GEMM for sm_100a.
//
// Computes C = alpha * op(A) * op(B) + beta * C, column-major, for
//   f16 x f16 -> f32 / f16 and bf16 x bf16 -> f32 / bf16  (tcgen05.mma kind::f16)
//   s8 x s8 -> s32                                         (tcgen05.mma kind::i8)
//   split f32 (FAST_TF32, see tf32_split.cu) -> f32          (tcgen05.mma kind::tf32)
// It replaces slang-gemm's cooperative-matrix shaders
// (shaders/gemm_nvcoop2_f16.slang, shaders/gemm_nvcoop2_i8.slang and the bf16
// path of tools/emit_nvcoop2_spv.zig); the arithmetic contract is gemmExCuda
// (src/gemm.zig:671-706).
//
// Design (persistent over output tiles, one CTA per SM):
//  - CG = 2 (default for M > 128): a cluster of two CTAs computes a 256 x 256
//    tile with tcgen05.mma.cta_group::2. Each CTA loads 128 rows of A and 128
//    of the 256 B columns, so per-SM operand traffic is 2/3 of the 1-SM tile;
//    the wide variant (long K loops) computes 256 x 512 with two such MMAs per
//    K step into all 512 TMEM columns, cutting operand traffic by another 1/4;
//    CG = 1: one CTA computes a 128 x 256 tile;
//  - 128 bytes of K per pipeline stage (64 f16/bf16, 128 s8 or 32 tf32), 6
//    stages (CG 2) or 4 stages (CG 1 and the wide pair tile);
//  - tf32 accumulates its K loop in fills of CHUNK_KB stages that the epilogue
//    folds into a running sum in the second TMEM half with exact f32 adds (the
//    tensor core's accumulation loses part of an ulp per step);
//  - warp 0: TMA producer. Operand transposes live in the tensor maps: op(A)=N
//    (M-contiguous) and op(B)=T (N-contiguous) are fetched as MN-major 128-byte
//    swizzled panels, op(A)=T and op(B)=N as K-major panels, and the UMMA
//    instruction descriptor's major bits tell the tensor core which is which;
//  - warp 1: allocates 512 TMEM columns (two 128 x 256 f32/s32 accumulators)
//    and, in the even CTA only, issues tcgen05.mma from one thread;
//    tcgen05.commit frees shared-memory stages and publishes accumulators
//    (to both CTAs of the pair for CG 2);
//  - warps 2..9 (2..17 for the wide tile): epilogue, two (four) warps per
//    TMEM lane quadrant, each draining half (a quarter) of a 256-column
//    accumulator (the wide tile's two halves in turn). tcgen05.ld gives each thread one
//    accumulator row; with beta == 0 a warp stages 32 rows x 16 columns in
//    shared memory (column-major, like C) and writes them with a TMA tensor
//    store (L2 evict_first); otherwise the 32 lanes store 32 consecutive rows
//    of one column directly. Double-buffered TMEM lets the epilogue of tile i
//    overlap the main loop of tile i+1.
// Batches (strided or pointer-array) are the outermost tile coordinate; the
// M/N tiles of one batch are visited in groups of `group_m` row blocks so
// that concurrently running CTAs share A and B panels in L2.
#include <cstdio>

#include "gs_epilogue.cuh"
#include "gs_internal.h"
#include "gs_ptx.cuh"
#include "gs_simt.cuh"

namespace gs {
namespace tc {

constexpr int BM = 128;        // accumulator rows per CTA
constexpr int BN = 256;        // accumulator columns per tcgen05.mma (and per tile unless wide)
constexpr int BK_BYTES = 128;  // K bytes per stage
constexpr int CHUNK_KB = 36;   // TF32: stages per accumulator fill (1152 K elements, 144 tcgen05.mma)
constexpr int TMEM_COLS = 2 * BN;
// Result stores are streamed through L2 (evict_first) so the output does not
// push operand panels out; operand loads of a single GEMM are kept
// (evict_last: its A and B panels are re-read by many tiles), those of batched
// calls use the normal policy (each batch entry's panels are short-lived).

// WIDE (CG 2 only): the pair computes a 256 x 512 tile as two 256 x 256
// tcgen05.mma per K step into one accumulator spanning all 512 TMEM columns.
// A is then reused over twice the columns: 48 KiB of operands per 1024
// tensor-core cycles instead of 32 KiB per 512, i.e. 3/4 of the L2 -> SM
// traffic (and power) of the 256 x 256 tile. The price is the single
// accumulator: the epilogue drains it in two 256-column halves, and the next
// tile's MMAs into a half wait until that half is drained.
template <int CG, bool WIDE>
struct Cfg {
    static constexpr int TILE_N = WIDE ? 2 * BN : BN;      // columns of one tile
    static constexpr int NSUB = TILE_N / BN;               // tcgen05.mma per K step
    // Epilogue warps: EPI_WARPS / 4 per TMEM lane quadrant, each draining EPI_COLS
    // columns of an accumulator slot. The wide tile's MMAs wait for its drain,
    // so it gets twice the warps (it has the registers: no CUDA-core fallback).
    static constexpr int EPI_WARPS = WIDE ? 16 : 8;
    static constexpr int EPI_COLS = BN / (EPI_WARPS / 4);
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int STAGES = WIDE ? 4 : (CG == 2 ? 6 : 4);
    static constexpr int B_BOX = BN / CG;                  // B columns per TMA box (one per sub-MMA)
    static constexpr int B_ROWS = NSUB * B_BOX;            // B columns this CTA loads per tile
    static constexpr int A_STAGE = BM * BK_BYTES;          // 16 KiB
    static constexpr int B_SUB = B_BOX * BK_BYTES;         // bytes of one B box
    static constexpr int B_STAGE = B_ROWS * BK_BYTES;      // 16 KiB (CG 2) / 32 KiB (CG 1, CG 2 wide)
    static constexpr int STAGE = A_STAGE + B_STAGE;
    static constexpr int TILE_M = BM * CG;                 // rows of one (pair) tile
    // Epilogue staging for TMA stores: per epilogue warp NSTG 32-row x 16-column x 4-byte blocks
    // (the wide tile's 16 warps get one each, which keeps its four operand stages).
    static constexpr int STG_BLOCK = 32 * 16 * 4;
    static constexpr int NSTG = WIDE ? 1 : 2;
    static constexpr int STG_BYTES = EPI_WARPS * NSTG * STG_BLOCK;
    static constexpr int SMEM = STAGES * STAGE + STG_BYTES + 1024 /*alignment slack*/ + 256 /*barriers*/;
};

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
    const uint32_t *skip_flag;   // pointer-array batches: == skip_gen when a pointer is not 16-byte aligned
    uint32_t skip_gen;
    const CUtensorMap *c_maps;   // pointer-array batches with TMA-stored C: per-batch C maps in global memory
    CUtensorMap *cta_maps;       // small pointer-array batches: per-CTA map slots (3 x batch each) that every CTA
                                 // fills itself from the templates tmA/tmB/tmC and args.fb's pointer arrays
    const uint32_t *c_skip_flag; // == skip_gen when a C pointer is not 16-byte aligned (C then stored directly)
    int tma_store;               // epilogue writes C with TMA tensor stores (beta == 0, C TMA-addressable)
    int ab_evict_last;           // operand loads use the evict_last L2 policy
    simt::SimtArgs fb;           // pointer-array batches: the CUDA-core fallback's view of the problem
    Epilogue ep;
    uint32_t *err;
    long long spin_limit;        // SM cycles after which a bounded wait gives up
    int debug_skip_kb;           // test hook (>= 0): the producer skips this K block of its first tile, then stops
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

template <int IN, int OUT, int CG, bool WIDE>
__global__ void __launch_bounds__(Cfg<CG, WIDE>::THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, const TcArgs args) {
    using C_ = Cfg<CG, WIDE>;
    static_assert(!WIDE || CG == 2, "the wide tile is a CTA-pair tile");
    constexpr int STAGES = C_::STAGES;
    constexpr int TILE_N = C_::TILE_N;
    constexpr int ES = (IN == IN_I8) ? 1 : (IN == IN_TF32 ? 4 : 2);  // element bytes
    constexpr int BK = BK_BYTES / ES;                  // K elements per stage
    constexpr int UK = 32 / ES;                        // K per tcgen05.mma (32 bytes)
    constexpr int CH = BK_BYTES / ES;                  // MN elements per 128-byte swizzle panel
    constexpr uint32_t CH_BYTES = CH * BK * ES;        // bytes of one MN-major panel (BK rows x 128 B)
    constexpr uint32_t C_FMT = (IN == IN_I8) ? 2u : 1u;
    constexpr uint32_t AB_FMT = (IN == IN_F16) ? 0u : (IN == IN_TF32 ? 2u : 1u);  // bf16 = 1, s8 = 1, tf32 = 2
    // TF32 (the split FAST_TF32 operands): the tensor core's f32 accumulation
    // loses a fraction of an ulp toward zero per accumulate step, so K is
    // accumulated in chunks of CHUNK_KB stages in TMEM columns [0, 256) and the
    // epilogue adds each chunk into a running sum in columns [256, 512) with
    // exact f32 adds; only the last chunk's sum is stored. Problems of a
    // single fill keep the usual double-buffered accumulators. The wide tile
    // has no second half to spare: it takes tf32 problems of a single fill only.
    constexpr bool CHUNKED = IN == IN_TF32 && !WIDE;
    const bool chunked = CHUNKED && args.k_blocks > CHUNK_KB;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *smA = smem;
    uint8_t *smB = smem + STAGES * C_::A_STAGE;
    uint8_t *stg = smB + STAGES * C_::B_STAGE;
    uint64_t *full = reinterpret_cast<uint64_t *>(stg + C_::STG_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;  // the MMA issuer's last commit on an error path
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;  // position in the CTA pair
    const bool leader = rank == 0;

    grid_dep_wait();
    grid_dep_launch();
    const CUtensorMap *a_maps = args.a_maps, *b_maps = args.b_maps, *c_maps = args.c_maps;
    // TMA-stored C; pointer-array batches fall back to direct stores when a C entry is misaligned.
    bool c_tma = args.tma_store && !(args.c_skip_flag != nullptr && *args.c_skip_flag == args.skip_gen);
    // Pointer-array batches whose pointers TMA cannot address: every CTA sees
    // the same answer and, instead of the tensor-core pipeline, runs the CUDA-core
    // tile loop over the whole batch (both CTAs of a pair take the same path,
    // before any cluster barrier or TMEM allocation).
    if constexpr (!WIDE && IN != IN_TF32) {  // pointer-array batches never use the wide tile or tf32
        if (args.cta_maps != nullptr) {
            // Small batches, one launch: the CTA checks every entry's pointers, then writes the maps it
            // uses into its own slots -- the template with the entry's address swapped in by
            // tensormap.replace -- and releases them to the tensor-map proxy; the threads that issue TMA
            // through a map acquire it first. Slots are private to the CTA, so no CTA waits for another.
            bool bad_ab = false, bad_c = false;
            for (int i = threadIdx.x; i < args.batch; i += blockDim.x) {
                const uint64_t pa = reinterpret_cast<uint64_t>(args.fb.a_arr[i]);
                const uint64_t pb = reinterpret_cast<uint64_t>(args.fb.b_arr[i]);
                bad_ab |= ((pa | pb) & 15u) != 0u;
                if (args.tma_store) bad_c |= (reinterpret_cast<uint64_t>(args.fb.c_arr[i]) & 15u) != 0u;
            }
            bad_ab = __syncthreads_or(bad_ab) != 0;
            bad_c = __syncthreads_or(bad_c) != 0;
            if (bad_ab) {
                simt::simt_tiles<IN, OUT>(args.fb, blockIdx.x, gridDim.x, smem);
                return;
            }
            c_tma = args.tma_store && !bad_c;
            CUtensorMap *own = args.cta_maps + static_cast<size_t>(blockIdx.x) * 3u * static_cast<size_t>(args.batch);
            for (int i = threadIdx.x; i < args.batch; i += blockDim.x) {
                own[i] = tmA;
                tensormap_set_address(own + i, args.fb.a_arr[i]);
                own[args.batch + i] = tmB;
                tensormap_set_address(own + args.batch + i, args.fb.b_arr[i]);
                if (c_tma) {
                    own[2 * args.batch + i] = tmC;
                    tensormap_set_address(own + 2 * args.batch + i, args.fb.c_arr[i]);
                }
            }
            tensormap_release();
            a_maps = own;
            b_maps = own + args.batch;
            c_maps = c_tma ? own + 2 * args.batch : nullptr;
        } else if (args.skip_flag != nullptr && *args.skip_flag == args.skip_gen) {
            simt::simt_tiles<IN, OUT>(args.fb, blockIdx.x, gridDim.x, smem);
            return;
        }
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            // One elected lane per epilogue warp (of both CTAs for CG 2).
            mbar_init(&tempty[i], CG * C_::EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0 && a_maps == nullptr) {
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        if constexpr (CG == 2) {
            tmem_alloc_2sm(tmem_holder, TMEM_COLS);
            tmem_relinquish_2sm();
        } else {
            tmem_alloc(tmem_holder, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    const long long tile0 = CG == 2 ? (blockIdx.x >> 1) : blockIdx.x;
    const long long tile_step = CG == 2 ? (gridDim.x >> 1) : gridDim.x;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            const uint64_t pol_ab = args.ab_evict_last ? l2_policy_evict_last() : l2_policy_evict_normal();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (long long t = tile0; ok && t < args.total_tiles; t += tile_step) {
                int b, mb, nb;
                tile_coords(args, t, b, mb, nb);
                const int m0 = mb * C_::TILE_M + static_cast<int>(rank) * BM;
                // B box s feeds sub-MMA s (tile columns s*256 .. s*256+255); of those,
                // this CTA of the pair holds columns rank*B_BOX .. rank*B_BOX+B_BOX-1.
                const int n0 = nb * TILE_N + static_cast<int>(rank) * C_::B_BOX;
                const CUtensorMap *ma = &tmA, *mbp = &tmB;
                int ab = args.a_bcast ? 0 : b, bb = args.b_bcast ? 0 : b;
                if (a_maps != nullptr) {
                    ma = a_maps + b;
                    mbp = b_maps + b;
                    ab = 0;
                    bb = 0;
                    tensormap_acquire(ma);
                    tensormap_acquire(mbp);
                }
                for (int kb = 0; kb < args.k_blocks; ++kb) {
                    // Test hook: leave this stage unfilled (no expect_tx, no copy) and issue nothing more, so
                    // the MMA issuer's wait for it runs out with no load left in flight.
                    if (kb == args.debug_skip_kb && t == tile0) { ok = false; break; }
                    if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, 1, args.spin_limit)) { ok = false; break; }
                    uint8_t *dA = smA + stage * C_::A_STAGE;
                    uint8_t *dB = smB + stage * C_::B_STAGE;
                    const int k0 = kb * BK;
                    if constexpr (CG == 2) {
                        // Both CTAs' bytes complete on the even CTA's barrier.
                        const uint32_t fbar = mapa_shared(smem_u32(&full[stage]), 0);
                        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C_::STAGE);
                        if (args.a_mn) {
#pragma unroll
                            for (int c = 0; c < BM / CH; ++c)
                                tma_load_3d_2sm(dA + c * CH_BYTES, ma, fbar, m0 + c * CH, k0, ab, pol_ab);
                        } else {
                            tma_load_3d_2sm(dA, ma, fbar, k0, m0, ab, pol_ab);
                        }
#pragma unroll
                        for (int s = 0; s < C_::NSUB; ++s) {
                            uint8_t *dBs = dB + s * C_::B_SUB;
                            const int ns = n0 + s * BN;
                            if (args.b_mn) {
#pragma unroll
                                for (int c = 0; c < C_::B_BOX / CH; ++c)
                                    tma_load_3d_2sm(dBs + c * CH_BYTES, mbp, fbar, ns + c * CH, k0, bb, pol_ab);
                            } else {
                                tma_load_3d_2sm(dBs, mbp, fbar, k0, ns, bb, pol_ab);
                            }
                        }
                    } else {
                        mbar_arrive_expect_tx(&full[stage], C_::STAGE);
                        if (args.a_mn) {
#pragma unroll
                            for (int c = 0; c < BM / CH; ++c)
                                tma_load_3d_hint(dA + c * CH_BYTES, ma, &full[stage], m0 + c * CH, k0, ab, pol_ab);
                        } else {
                            tma_load_3d_hint(dA, ma, &full[stage], k0, m0, ab, pol_ab);
                        }
                        if (args.b_mn) {
#pragma unroll
                            for (int c = 0; c < C_::B_ROWS / CH; ++c)
                                tma_load_3d_hint(dB + c * CH_BYTES, mbp, &full[stage], n0 + c * CH, k0, bb, pol_ab);
                        } else {
                            tma_load_3d_hint(dB, mbp, &full[stage], k0, n0, bb, pol_ab);
                        }
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA only) ----------------
        if (lane == 0 && leader) {
            const uint32_t idesc = umma_idesc(C_FMT, AB_FMT, args.a_mn, args.b_mn, C_::TILE_M, BN);
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            // Accumulator slots: two 256-column buffers used by alternate tiles, or
            // (WIDE) the two halves of one 512-column accumulator used by every tile.
            auto commit_to = [&](uint64_t *bar) {
                if constexpr (CG == 2) umma_commit_2sm(bar, 0x3);
                else umma_commit(bar);
            };
            uint32_t chunks = 0;  // CHUNKED: accumulator fills issued so far
            for (long long t = tile0; ok && t < args.total_tiles; t += tile_step, ++it) {
                const int acc = (WIDE || chunked) ? 0 : (it & 1);
                const uint32_t acc_phase = WIDE ? (it & 1) : ((it >> 1) & 1);
                if (!chunked) {
                    if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.err, 2, args.spin_limit)) { ok = false; break; }
                    tc_fence_after();
                }
                const uint32_t d_tmem = tmem_base + acc * BN;
                // One K step of sub-MMA s from stage st into accumulator columns s*BN..;
                // `first` starts the accumulation (the first K step of a tile or fill).
                auto issue = [&](int st, int s, bool first) {
                    const uint32_t a_base = smem_u32(smA + st * C_::A_STAGE);
                    const uint32_t b_base = smem_u32(smB + st * C_::B_STAGE + s * C_::B_SUB);
#pragma unroll
                    for (int kk = 0; kk < BK / UK; ++kk) {
                        const uint64_t adesc = args.a_mn
                                                   ? umma_smem_desc_sw128(a_base + kk * UK * 128, CH_BYTES, 1024)
                                                   : umma_smem_desc_sw128(a_base + kk * UK * ES, 16, 1024);
                        const uint64_t bdesc = args.b_mn
                                                   ? umma_smem_desc_sw128(b_base + kk * UK * 128, CH_BYTES, 1024)
                                                   : umma_smem_desc_sw128(b_base + kk * UK * ES, 16, 1024);
                        const uint32_t accum = (!first || kk != 0) ? 1u : 0u;
                        const uint32_t d = d_tmem + s * BN;
                        if constexpr (CG == 2) {
                            if constexpr (IN == IN_I8) umma_i8_2sm(d, adesc, bdesc, idesc, accum);
                            else if constexpr (IN == IN_TF32) umma_tf32_2sm(d, adesc, bdesc, idesc, accum);
                            else umma_f16_2sm(d, adesc, bdesc, idesc, accum);
                        } else {
                            if constexpr (IN == IN_I8) umma_i8(d, adesc, bdesc, idesc, accum);
                            else if constexpr (IN == IN_TF32) umma_tf32(d, adesc, bdesc, idesc, accum);
                            else umma_f16(d, adesc, bdesc, idesc, accum);
                        }
                    }
                };
                int kb = 0;
                if constexpr (WIDE) {
                    // The second accumulator half is drained after the first, so the tile
                    // opens with the first half's MMAs over the stages already loaded, then
                    // waits for the second half and catches up on the same stages.
                    const int P = args.k_blocks < STAGES ? args.k_blocks : STAGES;
                    int st = stage;
                    uint32_t ph = phase;
                    for (int j = 0; j < P; ++j) {
                        if (!mbar_wait(&full[st], ph, args.err, 3, args.spin_limit)) { ok = false; break; }
                        tc_fence_after();
                        issue(st, 0, j == 0);
                        if (j + 1 == args.k_blocks) commit_to(&tfull[0]);
                        if (++st == STAGES) { st = 0; ph ^= 1u; }
                    }
                    if (!ok) break;
                    if (!mbar_wait(&tempty[1], acc_phase ^ 1u, args.err, 2, args.spin_limit)) { ok = false; break; }
                    tc_fence_after();
                    for (int j = 0; j < P; ++j) {
                        issue(stage, 1, j == 0);
                        commit_to(&empty[stage]);
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                    kb = P;
                }
                // WIDE with a long K loop: the last `tail` K steps run as all first-half
                // MMAs, then all second-half ones, so the first half is published (and
                // drains) while the second half's last MMAs run. (Short loops lose more
                // to the stages held back meanwhile: C4's 16 K steps measured 3 % slower.)
                const int tail = (WIDE && args.k_blocks >= 32)
                                     ? (args.k_blocks - kb < STAGES ? args.k_blocks - kb : STAGES)
                                     : 0;
                for (; kb < args.k_blocks - tail; ++kb) {
                    const int kb_in = chunked ? kb % CHUNK_KB : kb;  // stage within the accumulator fill
                    if (chunked && kb_in == 0) {
                        // the epilogue has folded the previous fill into the running sum
                        if (!mbar_wait(&tempty[0], (chunks & 1u) ^ 1u, args.err, 2, args.spin_limit)) { ok = false; break; }
                        tc_fence_after();
                    }
                    if (!mbar_wait(&full[stage], phase, args.err, 3, args.spin_limit)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int s = 0; s < C_::NSUB; ++s) {
                        issue(stage, s, kb_in == 0);
                        // Last K step: publish the first half as soon as its MMAs are issued,
                        // so its drain overlaps the second half's last MMAs.
                        if (WIDE && s == 0 && kb + 1 == args.k_blocks) commit_to(&tfull[0]);
                    }
                    commit_to(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    if (chunked && (kb_in == CHUNK_KB - 1 || kb + 1 == args.k_blocks)) {
                        commit_to(&tfull[0]);
                        ++chunks;
                    }
                }
                if (WIDE && ok && tail > 0) {
                    int st = stage;
                    uint32_t ph = phase;
                    for (int j = 0; j < tail; ++j) {
                        if (!mbar_wait(&full[st], ph, args.err, 3, args.spin_limit)) { ok = false; break; }
                        tc_fence_after();
                        issue(st, 0, false);
                        if (++st == STAGES) { st = 0; ph ^= 1u; }
                    }
                    if (!ok) break;
                    commit_to(&tfull[0]);
                    for (int j = 0; j < tail; ++j) {
                        issue(stage, 1, false);
                        commit_to(&empty[stage]);
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                }
                if (ok && !chunked) commit_to(&tfull[WIDE ? 1 : acc]);
            }
            if (!ok) {
                // A wait gave up: before the CTA tears down (and frees TMEM), wait, again within the limit,
                // until the MMAs already issued have completed.
                commit_to(drain);
                mbar_wait(drain, 0, args.err, 5, args.spin_limit);
            }
        }
    } else {
        // ---------------- epilogue warps 2..2+EPI_WARPS-1 (both CTAs) ----------------
        const int quad = warp & 3;                  // TMEM lane quadrant this warp may access
        const int ew = warp - 2;                    // epilogue warp index
        const int c_lo = (ew / 4) * C_::EPI_COLS;   // this warp's share of the accumulator columns
        const int row = quad * 32 + lane;
        const uint32_t tempty_leader = CG == 2 ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;
        const uint64_t pol_c = l2_policy_evict_first();
        int stg_flip = 0;
        int it = 0;
        uint32_t echunks = 0;  // CHUNKED: accumulator fills consumed so far
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
        auto arrive_tempty = [&](int acc) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 2) mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
                else mbar_arrive(&tempty[acc]);
            }
        };
        bool ok = true;
        for (long long t = tile0; ok && t < args.total_tiles; t += tile_step, ++it) {
            int b, mb, nb;
            tile_coords(args, t, b, mb, nb);
            const int m = mb * C_::TILE_M + static_cast<int>(rank) * BM + row;
            const int nfills = chunked ? (args.k_blocks + CHUNK_KB - 1) / CHUNK_KB : 1;
            if constexpr (CHUNKED) {
                // Fold every fill but the last into the running sum (columns BN..2BN-1), in order.
#pragma unroll 1
                for (int f = 0; ok && f + 1 < nfills; ++f) {
                    // every lane of the warp takes the same way out (tcgen05.ld below is warp-aligned)
                    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[0], echunks & 1u, args.err, 4, args.spin_limit))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = c_lo; c < c_lo + C_::EPI_COLS; c += 32) {
                        uint32_t r[32], sum[32];
                        tmem_ld_32x32b_x32(t_lane + c, r);
                        if (f > 0) tmem_ld_32x32b_x32(t_lane + BN + c, sum);
                        tmem_wait_ld();
                        if (f > 0) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                r[j] = __float_as_uint(__fadd_rn(__uint_as_float(sum[j]), __uint_as_float(r[j])));
                        }
                        tmem_st_32x32b_x32(t_lane + BN + c, r);
                    }
                    tmem_wait_st();
                    arrive_tempty(0);
                    ++echunks;
                }
                if (!ok) break;
            }
            void *Cb = args.C;
            if (args.c_arr != nullptr) Cb = args.c_arr[b];
            else Cb = static_cast<uint8_t *>(args.C) + static_cast<size_t>(b) * args.stride_c *
                                                        ((OUT == OUT_F16 || OUT == OUT_BF16) ? 2 : 4);
            const CUtensorMap *cmap = c_maps != nullptr ? c_maps + b : &tmC;
            const int cz = c_maps != nullptr ? 0 : b;
            if (c_tma && c_maps != nullptr && lane == 0) tensormap_acquire(cmap);
            // One pass per accumulator slot this tile owns: the tile's 256-column
            // buffer, or (WIDE) each half of the 512-column accumulator in turn.
#pragma unroll 1
            for (int half = 0; half < C_::NSUB; ++half) {
            const int acc = WIDE ? half : (chunked ? 0 : (it & 1));
            const uint32_t acc_phase = chunked ? (echunks & 1u) : (WIDE ? (it & 1) : ((it >> 1) & 1));
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, args.err, 4, args.spin_limit))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int n0 = nb * TILE_N + half * BN;  // tile column of this slot's first accumulator column
            const int ncols = min(BN, args.n - n0);
#pragma unroll 1
            for (int c = c_lo; c < c_lo + C_::EPI_COLS; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_lane + acc * BN + c, r);
                if (chunked && nfills > 1) {
                    uint32_t sum[32];
                    tmem_ld_32x32b_x32(t_lane + BN + c, sum);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        r[j] = __float_as_uint(__fadd_rn(__uint_as_float(sum[j]), __uint_as_float(r[j])));
                } else {
                    tmem_wait_ld();
                }
                if (c_tma) {
                    // Stage this warp's 32 rows in blocks of 16 columns (column-major, like C)
                    // and write each block with one TMA tensor store; edge elements are
                    // clipped by TMA. Two staging buffers per warp alternate.
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (c + 16 * h >= ncols) continue;
                        uint8_t *buf = stg + (ew * C_::NSTG + stg_flip) * C_::STG_BLOCK;
                        stg_flip = stg_flip + 1 == C_::NSTG ? 0 : stg_flip + 1;
                        if (lane == 0) bulk_wait_group_read<C_::NSTG - 1>();  // the store that last used `buf` has read it
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const uint32_t raw = r[16 * h + j];
                            if constexpr (OUT == OUT_I32) {
                                int32_t v = static_cast<int32_t>(raw);
                                if (!args.ep.identity) {
                                    double t = __dmul_rn(static_cast<double>(args.ep.alpha_i), static_cast<double>(v));
                                    t = fmin(2147483647.0, fmax(-2147483648.0, round(t)));
                                    v = static_cast<int32_t>(t);
                                }
                                reinterpret_cast<int32_t *>(buf)[j * 32 + lane] = v;
                            } else {
                                float v = __uint_as_float(raw);
                                if (!args.ep.identity) v = args.ep.alpha_f * v;
                                if constexpr (OUT == OUT_F32) reinterpret_cast<float *>(buf)[j * 32 + lane] = v;
                                else if constexpr (OUT == OUT_F16) reinterpret_cast<__half *>(buf)[j * 32 + lane] = __float2half_rn(v);
                                else reinterpret_cast<uint16_t *>(buf)[j * 32 + lane] = bf16_bits_ref_round(v);
                            }
                        }
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_3d(cmap, buf, mb * C_::TILE_M + static_cast<int>(rank) * BM + quad * 32,
                                         n0 + c + 16 * h, cz, pol_c);
                            bulk_commit_group();
                        }
                    }
                    continue;
                }
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
            arrive_tempty(acc);
            if (chunked) ++echunks;
            }  // accumulator slots of this tile
        }
        if (c_tma && lane == 0) bulk_wait_group_all();  // C is written before the kernel ends
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();  // neither CTA leaves while the peer may still signal its barriers
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (CG == 2) tmem_dealloc_2sm(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Kernel that writes one tensor map per pointer-array batch entry: it copies
// a host-encoded template and patches the global address with
// tensormap.replace, then makes the write visible to the tensor-map proxy.
// A pointer that is not 16-byte aligned cannot be a TMA base address: the
// builder then writes this call's tag `gen` into *misaligned and the
// tensor-core kernel computes the whole batch with its CUDA-core fallback
// instead (a word tagged by an earlier call never matches). C maps (written
// when maps_c is not null) have their own flag: a misaligned C entry only
// switches the epilogue to direct stores.
__global__ void k_build_ptr_maps(const CUtensorMap tmpl_a, const CUtensorMap tmpl_b, const CUtensorMap tmpl_c,
                                 const void *const *a_arr, const void *const *b_arr, void *const *c_arr,
                                 CUtensorMap *maps_a, CUtensorMap *maps_b, CUtensorMap *maps_c, int batch,
                                 uint32_t *misaligned, uint32_t *misaligned_c, uint32_t gen) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch) return;
    if (maps_c != nullptr) {
        const uint64_t pc = reinterpret_cast<uint64_t>(c_arr[i]);
        if ((pc & 15u) != 0u) {
            atomicExch(misaligned_c, gen);
        } else {
            maps_c[i] = tmpl_c;
            tensormap_set_address(maps_c + i, c_arr[i]);
        }
    }
    const uint64_t pa = reinterpret_cast<uint64_t>(a_arr[i]), pb = reinterpret_cast<uint64_t>(b_arr[i]);
    if (((pa | pb) & 15u) != 0u) {
        atomicExch(misaligned, gen);
        return;
    }
    maps_a[i] = tmpl_a;
    maps_b[i] = tmpl_b;
    tensormap_set_address(maps_a + i, a_arr[i]);
    tensormap_set_address(maps_b + i, b_arr[i]);
    tensormap_release();
}

// Largest number of co-resident CTA pairs for one 2-SM kernel instantiation on this device.
template <int IN, int OUT, int CG, bool WIDE>
static int max_pairs(Context &ctx) {
    using C_ = Cfg<CG, WIDE>;
    auto kern = k_gemm_tc<IN, OUT, CG, WIDE>;
    static int cached[64] = {};  // per instantiation and device
    if (ctx.device >= 0 && ctx.device < 64 && cached[ctx.device] > 0) return cached[ctx.device];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (ctx.sm_count / 2), 1, 1);
    cfg.blockDim = dim3(C_::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C_::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = ctx.sm_count / 2;
    }
    if (ctx.device >= 0 && ctx.device < 64) cached[ctx.device] = n;
    return n;
}

template <int IN, int OUT, int CG, bool WIDE>
static cudaError_t launch_kernel(Context &ctx, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tcm,
                                 const TcArgs &args) {
    using C_ = Cfg<CG, WIDE>;
    auto kern = k_gemm_tc<IN, OUT, CG, WIDE>;
    static bool attr_set[64] = {};  // per instantiation and device
    cudaError_t e = cudaSuccess;
    if (ctx.device < 0 || ctx.device >= 64 || !attr_set[ctx.device]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM);
        if (e != cudaSuccess) return e;
        if (ctx.device >= 0 && ctx.device < 64) attr_set[ctx.device] = true;
    }
    if constexpr (CG == 2) {
        const long long mp = max_pairs<IN, OUT, CG, WIDE>(ctx);
        const long long pairs = args.total_tiles < mp ? args.total_tiles : mp;
        if (args.cta_maps != nullptr && 2 * pairs > ctx.sm_count) return cudaErrorInvalidConfiguration;  // slots per CTA
        e = launch_pdl(kern, dim3(static_cast<unsigned>(2 * pairs)), dim3(C_::THREADS), C_::SMEM, ctx.stream, 2, ta,
                       tb, tcm, args);
        ctx.launches++;
        return e;
    } else {
        const long long grid = args.total_tiles < ctx.sm_count ? args.total_tiles : ctx.sm_count;
        e = launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(C_::THREADS), C_::SMEM, ctx.stream, 1, ta, tb,
                       tcm, args);
        ctx.launches++;
        return e;
    }
}

template <int CG, bool WIDE>
static cudaError_t dispatch(Context &ctx, const GemmDesc &d, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tcm,
                            const TcArgs &args) {
    switch (d.in_kind) {
    case IN_F16:
        if (d.out_kind == OUT_F32) return launch_kernel<IN_F16, OUT_F32, CG, WIDE>(ctx, ta, tb, tcm, args);
        if (d.out_kind == OUT_F16) return launch_kernel<IN_F16, OUT_F16, CG, WIDE>(ctx, ta, tb, tcm, args);
        break;
    case IN_BF16:
        if (d.out_kind == OUT_F32) return launch_kernel<IN_BF16, OUT_F32, CG, WIDE>(ctx, ta, tb, tcm, args);
        if (d.out_kind == OUT_BF16) return launch_kernel<IN_BF16, OUT_BF16, CG, WIDE>(ctx, ta, tb, tcm, args);
        break;
    case IN_I8:
        if (d.out_kind == OUT_I32) return launch_kernel<IN_I8, OUT_I32, CG, WIDE>(ctx, ta, tb, tcm, args);
        break;
    case IN_TF32:  // the wide tile only for a single accumulator fill (choose_shape)
        if (d.out_kind == OUT_F32) return launch_kernel<IN_TF32, OUT_F32, CG, WIDE>(ctx, ta, tb, tcm, args);
        break;
    default: break;
    }
    return cudaErrorInvalidValue;
}

// Tile shape: 1 = 128 x 256 (one SM), 2 = 256 x 256 (CTA pair), 3 = 256 x 512 (CTA pair, wide).
static cudaError_t dispatch_shape(int shape, Context &ctx, const GemmDesc &d, const CUtensorMap &ta,
                                  const CUtensorMap &tb, const CUtensorMap &tcm, const TcArgs &args) {
    if (shape == 3) return dispatch<2, true>(ctx, d, ta, tb, tcm, args);
    if (shape == 2) return dispatch<2, false>(ctx, d, ta, tb, tcm, args);
    return dispatch<1, false>(ctx, d, ta, tb, tcm, args);
}

static CUtensorMapDataType tmap_dtype(InKind k) {
    return k == IN_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
           : k == IN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
           : k == IN_TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : CU_TENSOR_MAP_DATA_TYPE_UINT8;
}

// Encodes the A and B maps. `batch_a`/`batch_b` are the extents of the third
// (batch) dimension: 1 when every batch entry reads the same matrix.
// `b_rows` is the number of B columns one CTA loads per tile (256 / CG).
static bool make_maps(const GemmDesc &d, const void *a_base, const void *b_base, int batch_a, int batch_b,
                      uint32_t b_rows, CUtensorMap *ta, CUtensorMap *tb, std::string *why) {
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
                        d.trans_b ? ch : bk, d.trans_b ? bk : b_rows, why))
        return false;
    return true;
}

// Encodes the tensor map the epilogue stores C through (32 x 32 boxes, no
// swizzle). Only for beta == 0 (C is not read) and a C that TMA can address:
// 16-byte aligned base, leading dimension and batch stride.
static bool make_c_map(const GemmDesc &d, CUtensorMap *tcm) {
    if (!d.ep.beta_zero) return false;
    const uint64_t es = out_elem_size(d.out_kind);
    if ((reinterpret_cast<uintptr_t>(d.C) & 15u) != 0 || (static_cast<uint64_t>(d.ldc) * es) % 16 != 0) return false;
    if (d.batch > 1 && (d.stride_c <= 0 || (static_cast<uint64_t>(d.stride_c) * es) % 16 != 0)) return false;
    const CUtensorMapDataType dt = d.out_kind == OUT_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : d.out_kind == OUT_I32 ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                   : d.out_kind == OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t s1 = static_cast<uint64_t>(d.ldc) * es;
    const uint64_t s2 = d.batch > 1 ? static_cast<uint64_t>(d.stride_c) * es : static_cast<uint64_t>(d.n) * s1;
    return encode_tmap_3d(tcm, dt, d.C, static_cast<uint64_t>(d.m), static_cast<uint64_t>(d.n),
                          static_cast<uint64_t>(d.batch), s1, s2, 32, 16, nullptr, CU_TENSOR_MAP_SWIZZLE_NONE);
}

static TcArgs make_args(Context &ctx, const GemmDesc &d, int shape) {
    const int cg = shape == 1 ? 1 : 2;
    const int es = static_cast<int>(in_elem_size(d.in_kind));
    const int bk = BK_BYTES / es;
    const int tile_m = BM * cg;
    const int tile_n = shape == 3 ? 2 * BN : BN;
    TcArgs a{};
    a.m = d.m;
    a.n = d.n;
    a.k = d.k;
    a.batch = d.batch;
    a.m_blocks = (d.m + tile_m - 1) / tile_m;
    a.n_blocks = (d.n + tile_n - 1) / tile_n;
    a.k_blocks = (d.k + bk - 1) / bk;
    a.tiles_per_batch = static_cast<long long>(a.m_blocks) * a.n_blocks;
    a.total_tiles = a.tiles_per_batch * d.batch;
    a.a_mn = d.trans_a ? 0 : 1;
    a.b_mn = d.trans_b ? 1 : 0;
    a.a_bcast = (d.batch == 1 || d.stride_a == 0) ? 1 : 0;
    a.b_bcast = (d.batch == 1 || d.stride_b == 0) ? 1 : 0;
    const int group = cg == 2 ? 8 : 16;
    a.group_m = a.m_blocks < group ? a.m_blocks : group;
    a.C = d.C;
    a.ldc = d.ldc;
    a.stride_c = d.stride_c;
    a.c_arr = nullptr;
    a.a_maps = nullptr;
    a.b_maps = nullptr;
    a.skip_flag = nullptr;
    a.ab_evict_last = d.batch == 1 ? 1 : 0;
    a.ep = d.ep;
    a.err = ctx.dev_err;
    a.spin_limit = ctx.spin_limit;
    a.debug_skip_kb = ctx.debug_skip_kb;
    return a;
}

// Tile-shape choice. The algo argument is honoured as a hint
// (CUBLAS_GEMM_ALGO0 = 1-SM 128 x 256 tile, ALGO1 = 2-SM 256 x 256 pair tile,
// ALGO2 = 2-SM 256 x 512 wide pair tile). Otherwise, from a timed sweep of
// every tile over 36 shapes x FP16 / INT8 (single GEMMs 1024^3 .. 16384 x 4096,
// K 256 .. 16384, batches of 8 .. 256):
//  - the persistent kernel runs its tiles in rounds over the resident CTAs
//    (148 one-SM CTAs or 74 pairs), so a shape costs about
//    rounds x (work per SM per tile) / (the tile's throughput): 128 x 256 x K
//    per SM for the 1-SM and pair tiles, 128 x 512 x K for the wide tile, at
//    throughputs 0.86 / 0.91 / 1 of the wide tile's (measured at 8192^3); the
//    cheapest wins;
//  - when every 1-SM tile fits in one round the 1-SM tile is taken: it then
//    ran 1-7 % ahead of the pair tile and up to 1.7x ahead of the wide one
//    (1024^3, 2048^3, 512 x 512 x 16384);
//  - with at most 4 K stages the call is all epilogue and the wide tile, whose
//    16 epilogue warps drain C fastest, is taken (INT8 8192 x 4096 x 256:
//    1.3x ahead of the pair tile);
//  - for 16-bit operands with 5-15 K stages the wide tile's cost carries its
//    exposed accumulator drain, (stages + 2) / stages.
// Against the earlier rule (wide tile for >= 32 K stages or below the
// tensor / HBM ridge) this took the sweep's geometric-mean loss against the
// best tile from 9.7 % to 0.4 %; every configuration of the north star keeps
// the wide tile.
static int choose_shape_any(const GemmDesc &d, long long pairs);
static int choose_shape(const Context &ctx, const GemmDesc &d) {
    const int shape = choose_shape_any(d, ctx.sm_count >= 2 ? ctx.sm_count / 2 : 1);
    // TF32 past one accumulator fill keeps a running sum in the second TMEM
    // half, which the wide tile occupies.
    const int k_blocks = (d.k + BK_BYTES / 4 - 1) / (BK_BYTES / 4);
    return shape == 3 && d.in_kind == IN_TF32 && k_blocks > CHUNK_KB ? 2 : shape;
}
static int choose_shape_any(const GemmDesc &d, long long pairs) {
    if (d.algo == 0) return 1;
    if (d.algo == 1) return 2;
    if (d.algo == 2) return 3;
    if (d.m <= BM) return 1;
    auto cdiv = [](long long x, long long y) { return (x + y - 1) / y; };
    const long long mb1 = cdiv(d.m, BM), mb2 = cdiv(d.m, 2 * BM);
    const long long t1 = mb1 * cdiv(d.n, BN) * d.batch;       // 128 x 256 tiles
    const long long t2 = mb2 * cdiv(d.n, BN) * d.batch;       // 256 x 256 pair tiles
    const long long t3 = mb2 * cdiv(d.n, 2 * BN) * d.batch;   // 256 x 512 wide tiles
    const long long r1 = cdiv(t1, 2 * pairs), r2 = cdiv(t2, pairs), r3 = cdiv(t3, pairs);
    if (r1 == 1) return 1;
    const int es = static_cast<int>(in_elem_size(d.in_kind));
    const int k_blocks = static_cast<int>(cdiv(d.k, BK_BYTES / es));
    if (d.n > BN && k_blocks <= 4) return 3;
    const double c1 = static_cast<double>(r1) / 0.86, c2 = static_cast<double>(r2) / 0.91;
    double c3 = 2.0 * static_cast<double>(r3);
    // 16-bit operands with fewer than 16 K stages: the wide tile's single accumulator leaves about two stages'
    // worth of drain exposed per tile (batched 512^3 x 64 and 512 x 1024 x 512 x 96 ran 8-17 % faster on the
    // pair tile; 4096^2 x 512 and 8192 x 2048 x 512 2 % slower).
    if ((d.in_kind == IN_F16 || d.in_kind == IN_BF16) && k_blocks < 16)
        c3 *= (static_cast<double>(k_blocks) + 2.0) / static_cast<double>(k_blocks);
    if (c3 <= c2 && c3 <= c1) return 3;
    return c1 < c2 ? 1 : 2;
}

}  // namespace tc

namespace tc {

// Split-K reduction: C = alpha * (sum over the K slices' partial results, in slice order) + beta * C, with the
// epilogue rounding of every other path. Partial slice s of element (row, col) is ws[s * m * n + col * m + row].
// With M a multiple of 4 each thread takes four consecutive rows of one column: 16-byte loads of the partials.
template <int OUT>
__global__ void k_splitk_reduce(const void *ws, int parts, int m, int n, void *C, long long ldc, Epilogue ep) {
    grid_dep_wait();
    grid_dep_launch();
    const size_t mn = static_cast<size_t>(m) * static_cast<size_t>(n);
    const size_t first = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t step = static_cast<size_t>(gridDim.x) * blockDim.x;
    if ((m & 3) == 0) {
        const size_t q = mn / 4;
        for (size_t v = first; v < q; v += step) {
            const size_t i = 4 * v, col = i / static_cast<size_t>(m), row = i - col * static_cast<size_t>(m);
            const size_t dst = row + col * static_cast<size_t>(ldc);
            // Loads go out four slices at a time, ahead of their adds (the sum stays in slice order).
            if constexpr (OUT == OUT_I32) {
                const int4 *p = static_cast<const int4 *>(ws) + v;
                int4 a = make_int4(0, 0, 0, 0);
                int s = 0;
                for (; s + 4 <= parts; s += 4) {
                    int4 t[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) t[j] = __ldcs(p + static_cast<size_t>(s + j) * q);
#pragma unroll
                    for (int j = 0; j < 4; ++j) { a.x += t[j].x; a.y += t[j].y; a.z += t[j].z; a.w += t[j].w; }
                }
                for (; s < parts; ++s) {
                    const int4 t = __ldcs(p + static_cast<size_t>(s) * q);
                    a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
                }
                store_iacc(C, dst, a.x, ep); store_iacc(C, dst + 1, a.y, ep);
                store_iacc(C, dst + 2, a.z, ep); store_iacc(C, dst + 3, a.w, ep);
            } else {
                const float4 *p = static_cast<const float4 *>(ws) + v;
                float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                int s = 0;
                for (; s + 4 <= parts; s += 4) {
                    float4 t[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) t[j] = __ldcs(p + static_cast<size_t>(s + j) * q);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        a.x = __fadd_rn(a.x, t[j].x); a.y = __fadd_rn(a.y, t[j].y);
                        a.z = __fadd_rn(a.z, t[j].z); a.w = __fadd_rn(a.w, t[j].w);
                    }
                }
                for (; s < parts; ++s) {
                    const float4 t = __ldcs(p + static_cast<size_t>(s) * q);
                    a.x = __fadd_rn(a.x, t.x); a.y = __fadd_rn(a.y, t.y);
                    a.z = __fadd_rn(a.z, t.z); a.w = __fadd_rn(a.w, t.w);
                }
                store_facc<OUT>(C, dst, a.x, ep); store_facc<OUT>(C, dst + 1, a.y, ep);
                store_facc<OUT>(C, dst + 2, a.z, ep); store_facc<OUT>(C, dst + 3, a.w, ep);
            }
        }
        return;
    }
    for (size_t i = first; i < mn; i += step) {
        const size_t col = i / static_cast<size_t>(m), row = i - col * static_cast<size_t>(m);
        const size_t dst = row + col * static_cast<size_t>(ldc);
        if constexpr (OUT == OUT_I32) {
            const int32_t *p = static_cast<const int32_t *>(ws) + i;
            int32_t acc = 0;  // |sum| <= 128 * 128 * K < 2^31 (K is checked on entry)
            for (int s = 0; s < parts; ++s) acc += __ldcs(p + static_cast<size_t>(s) * mn);
            store_iacc(C, dst, acc, ep);
        } else {
            const float *p = static_cast<const float *>(ws) + i;
            float acc = 0.0f;
            for (int s = 0; s < parts; ++s) acc = __fadd_rn(acc, __ldcs(p + static_cast<size_t>(s) * mn));
            store_facc<OUT>(C, dst, acc, ep);
        }
    }
}

// K slices for a single GEMM whose 128 x 256 tiles fill less than half the SMs but whose K loop is long:
// the largest power of two S <= 32 that divides the K stages, leaves every slice >= 16 stages and keeps
// S x pair tiles within the SM pairs, if it is at least 4. 1 = no split. The slices run as a strided batch of the tensor-core
// kernel on the pair tile (with every SM busy the 1-SM tile's operand traffic saturates L2) into a handle
// workspace of S partial C (f32, or s32 for INT8), then k_splitk_reduce adds them in order.
// 512 x 512 x 16384: 4 pair tiles on 74 pairs become 16 slices x 4 tiles.
static int splitk_parts(const Context &ctx, const GemmDesc &d) {
    if (d.batch != 1 || d.algo >= 0 || d.in_kind == IN_TF32 || !ctx.may_allocate || d.m <= BM) return 1;
    const int bk = BK_BYTES / static_cast<int>(in_elem_size(d.in_kind));
    if (d.k % bk != 0) return 1;
    const long long kb = d.k / bk;
    const long long tiles1 = static_cast<long long>((d.m + BM - 1) / BM) * ((d.n + BN - 1) / BN);
    const long long tiles2 = static_cast<long long>((d.m + 2 * BM - 1) / (2 * BM)) * ((d.n + BN - 1) / BN);
    const long long sms = ctx.sm_count > 0 ? ctx.sm_count : 148;
    if (2 * tiles1 > sms) return 1;
    int s = 1;
    while (s < 32 && 2 * s * tiles2 <= sms / 2 && kb % (2 * s) == 0 && kb / (2 * s) >= 16) s *= 2;
    return s >= 4 ? s : 1;  // two slices do not pay for the reduction (INT8 1024^2 x 4096: 7 % slower)
}

}  // namespace tc

static cudaError_t launch_tc_one(Context &ctx, const GemmDesc &d);

void plan_tc_tile(const GemmDesc &d, int sm_count, int *tile, int *k_slices) {
    using namespace tc;
    Context c;
    c.sm_count = sm_count;
    const int parts = splitk_parts(c, d);
    GemmDesc p = d;
    if (parts > 1) {
        p.k = d.k / parts;
        p.batch = parts;
        p.algo = 1;
    }
    *k_slices = parts;
    *tile = choose_shape(c, p);
}

cudaError_t launch_tc(Context &ctx, const GemmDesc &d) {
    using namespace tc;
    const int parts = splitk_parts(ctx, d);
    if (parts == 1) return launch_tc_one(ctx, d);
    const size_t es_p = 4;  // f32 or s32 partials
    const size_t mn = static_cast<size_t>(d.m) * static_cast<size_t>(d.n);
    const size_t need = mn * static_cast<size_t>(parts) * es_p;
    if (ctx.splitk_bytes < need) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(ctx.stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
            ctx.last_error = "the split-K workspace must grow, which cannot be captured: make one call of this "
                             "size before the stream capture";
            return cudaErrorStreamCaptureUnsupported;
        }
        const size_t bytes = need > 2 * ctx.splitk_bytes ? need : 2 * ctx.splitk_bytes;
        void *grown = nullptr;
        const cudaError_t e = cudaMalloc(&grown, bytes);
        if (e == cudaErrorMemoryAllocation) {
            cudaGetLastError();
            return launch_tc_one(ctx, d);  // no room: the unsplit launch needs no workspace
        }
        if (e != cudaSuccess) return e;
        if (ctx.splitk_buf) ctx.retired.push_back(ctx.splitk_buf);  // kernels in flight may still use it
        ctx.splitk_buf = grown;
        ctx.splitk_bytes = bytes;
    }
    // The slices as a strided batch: slice s reads K elements [s*Ks, (s+1)*Ks) -- columns of a stored
    // op-N A / op-T B, rows of an op-T A / op-N B -- and writes partial s, alpha 1, beta 0.
    const long long ks = d.k / parts;
    GemmDesc p = d;
    p.k = static_cast<int>(ks);
    p.batch = parts;
    p.stride_a = d.trans_a ? ks : ks * d.lda;
    p.stride_b = d.trans_b ? ks * d.ldb : ks;
    p.out_kind = d.in_kind == IN_I8 ? OUT_I32 : OUT_F32;
    p.C = ctx.splitk_buf;
    p.ldc = d.m;
    p.stride_c = static_cast<long long>(mn);
    p.ep = Epilogue{1.0f, 0.0f, 1, 0, 1, 1};
    p.algo = 1;  // pair tile
    cudaError_t e = launch_tc_one(ctx, p);
    if (e != cudaSuccess) return e;
    const int threads = 256;
    const long long want = (static_cast<long long>(mn) + threads - 1) / threads;
    const unsigned blocks = static_cast<unsigned>(want < 8LL * ctx.sm_count ? want : 8LL * ctx.sm_count);
    switch (d.out_kind) {
    case OUT_F32: e = launch_pdl(k_splitk_reduce<OUT_F32>, dim3(blocks), dim3(threads), 0, ctx.stream, 1,
                                 static_cast<const void *>(ctx.splitk_buf), parts, d.m, d.n, d.C, d.ldc, d.ep); break;
    case OUT_F16: e = launch_pdl(k_splitk_reduce<OUT_F16>, dim3(blocks), dim3(threads), 0, ctx.stream, 1,
                                 static_cast<const void *>(ctx.splitk_buf), parts, d.m, d.n, d.C, d.ldc, d.ep); break;
    case OUT_BF16: e = launch_pdl(k_splitk_reduce<OUT_BF16>, dim3(blocks), dim3(threads), 0, ctx.stream, 1,
                                  static_cast<const void *>(ctx.splitk_buf), parts, d.m, d.n, d.C, d.ldc, d.ep); break;
    case OUT_I32: e = launch_pdl(k_splitk_reduce<OUT_I32>, dim3(blocks), dim3(threads), 0, ctx.stream, 1,
                                 static_cast<const void *>(ctx.splitk_buf), parts, d.m, d.n, d.C, d.ldc, d.ep); break;
    default: return cudaErrorInvalidValue;
    }
    ctx.launches++;
    ctx.last_kernels |= GS_KERNEL_REDUCE;
    return e;
}

static cudaError_t launch_tc_one(Context &ctx, const GemmDesc &d) {
    using namespace tc;
    const int shape = choose_shape(ctx, d);
    const int cg = shape == 1 ? 1 : 2;
    TcArgs args = make_args(ctx, d, shape);
    CUtensorMap ta, tb;
    std::string why;
    if (!make_maps(d, d.A, d.B, args.a_bcast ? 1 : d.batch, args.b_bcast ? 1 : d.batch, BN / cg, &ta, &tb, &why)) {
        ctx.last_error = "tensor map encode failed: " + why;
        return cudaErrorInvalidValue;
    }
    CUtensorMap tcm = ta;  // placeholder when the epilogue stores directly
    args.tma_store = make_c_map(d, &tcm) ? 1 : 0;
    return dispatch_shape(shape, ctx, d, ta, tb, tcm, args);
}

cudaError_t launch_tc_ptr_array(Context &ctx, const GemmDesc &d, const void *const *a_arr, const void *const *b_arr,
                                void *const *c_arr) {
    using namespace tc;
    // The wide tile has no CUDA-core fallback for misaligned entries: pair tile instead.
    const int shape = choose_shape(ctx, d) == 3 ? 2 : choose_shape(ctx, d);
    const int cg = shape == 1 ? 1 : 2;
    TcArgs args = make_args(ctx, d, shape);
    // Template maps over a placeholder (16-byte aligned, never dereferenced
    // through the template) with the per-batch geometry; each batch entry's
    // address is swapped in on the device. Small batches (and a handle that
    // may allocate) do that inside the GEMM kernel, one launch: every CTA fills
    // its own 3 x batch slots (the grid never exceeds the SM count). Larger
    // batches run the builder kernel first, which fills 3 x batch slots once.
    const bool in_kernel = ctx.may_allocate && d.batch <= GS_PTR_MAPS_IN_KERNEL_MAX_BATCH;
    const size_t slots = in_kernel ? static_cast<size_t>(ctx.sm_count) * static_cast<size_t>(d.batch)
                                   : static_cast<size_t>(d.batch);
    const size_t need = 3 * slots * sizeof(CUtensorMap);
    if (ctx.tmap_bytes < need) {
        // Grow-only, checked before anything of this call is enqueued. The old buffer may still be read
        // by kernels in flight, so it is not freed here (cudaFree would synchronise the device): it is
        // retired and freed with the handle. The first allocation holds 1024 entries and growth at least
        // doubles, so the retired buffers together stay smaller than the live one.
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(ctx.stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
            ctx.last_error = "the pointer-array tensor-map buffer must grow, which cannot be captured: make one "
                             "call with this batch count before the stream capture";
            return cudaErrorStreamCaptureUnsupported;
        }
        size_t bytes = 3 * size_t(1024) * sizeof(CUtensorMap);
        if (bytes < 2 * ctx.tmap_bytes) bytes = 2 * ctx.tmap_bytes;
        if (bytes < need) bytes = need;
        void *grown = nullptr;
        cudaError_t e = cudaMalloc(&grown, bytes);
        if (e != cudaSuccess) return e;
        if (ctx.tmap_buf) ctx.retired.push_back(ctx.tmap_buf);
        ctx.tmap_buf = grown;
        ctx.tmap_bytes = bytes;
    }
    CUtensorMap ta, tb;
    std::string why;
    const void *placeholder = ctx.tmap_buf;
    if (!make_maps(d, placeholder, placeholder, 1, 1, BN / cg, &ta, &tb, &why)) {
        ctx.last_error = "tensor map encode failed: " + why;
        return cudaErrorInvalidValue;
    }
    // With beta == 0 C is written by TMA stores through per-entry maps (one
    // batch entry each) built next to A's and B's; otherwise directly.
    CUtensorMap tcm = ta;
    GemmDesc dc = d;
    dc.batch = 1;
    dc.C = ctx.tmap_buf;
    const bool c_tma = make_c_map(dc, &tcm);
    args.tma_store = c_tma ? 1 : 0;
    args.a_bcast = 1;
    args.b_bcast = 1;
    args.c_arr = c_arr;
    args.fb = simt::make_args(d, a_arr, b_arr, c_arr);
    if (in_kernel) {
        args.cta_maps = static_cast<CUtensorMap *>(ctx.tmap_buf);
        return dispatch_shape(shape, ctx, d, ta, tb, tcm, args);
    }
    CUtensorMap *maps_a = static_cast<CUtensorMap *>(ctx.tmap_buf);
    CUtensorMap *maps_b = maps_a + d.batch;
    CUtensorMap *maps_c = c_tma ? maps_b + d.batch : nullptr;
    uint32_t *misaligned = ctx.dev_err + 1;
    uint32_t *misaligned_c = ctx.dev_err + 2;
    const uint32_t gen = ctx.next_ptr_gen();
    const int threads = 128;
    cudaError_t e = launch_pdl(k_build_ptr_maps, dim3((d.batch + threads - 1) / threads), dim3(threads), 0, ctx.stream,
                               1, ta, tb, tcm, a_arr, b_arr, c_arr, maps_a, maps_b, maps_c, d.batch, misaligned,
                               misaligned_c, gen);
    ctx.launches++;
    ctx.last_kernels |= GS_KERNEL_TMAP;
    if (e != cudaSuccess) return e;
    args.a_maps = maps_a;
    args.b_maps = maps_b;
    args.skip_flag = misaligned;
    args.skip_gen = gen;
    args.c_maps = maps_c;
    args.c_skip_flag = c_tma ? misaligned_c : nullptr;
    return dispatch_shape(shape, ctx, d, ta, tb, tcm, args);
}

}  // namespace gs
