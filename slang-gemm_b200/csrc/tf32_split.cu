// tf32_split.cu -- COMPUTE_32F_FAST_TF32 on the tensor cores.
//
// The reference computes every gemmEx in f64 whatever compute type it is given
// (src/gemm.zig:671-706, compute_type ignored at :686), so an f32 result has to
// stay within the FP32 tolerance even when the caller allowed TF32. One tf32
// product per f32 product would not (about 1e-3 relative); three do. Each
// operand value x is split into hi = x with the low 13 mantissa bits cleared
// (tf32-exact) and lo = x - hi (exact in f32, itself rounded to tf32 by the
// tensor core), and
//     a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi
// with an error of about 2^-20 |a b| (the dropped a_lo*b_lo and the tf32
// rounding of the lo parts). The three products become ONE tcgen05 kind::tf32
// GEMM over a K three times as long: A' = [A_hi | A_hi | A_lo] and
// B' = [B_hi ; B_lo ; B_hi] along K, both written K-major into handle-owned
// memory by a transpose-capable split kernel, with one fp32 accumulator and
// the usual alpha/beta epilogue. Non-finite inputs are outside this scheme
// (an infinite x gives lo = NaN); COMPUTE_32F keeps the exact FFMA kernel.
//
// Measured against an f64 product (N(0,1) inputs, B200): with one accumulator
// the normwise error grows linearly with K, about 1.1e-8 * K (6.1e-6 at
// K = 512, 2.2e-5 at 2048, 8.6e-5 at 8192), while the split itself costs about
// 1e-6: it is the tensor core's f32 accumulation, which loses a fraction of an
// ulp toward zero at every accumulate step, so the error tracks the number of
// steps. The GEMM kernel therefore accumulates its IN_TF32 K loop in fills of
// 36 stages (1152 elements of the 3K axis, like one K = 384 GEMM: ~4.7e-6) and
// adds the fills in TMEM with exact f32 adds (gemm_tc_sm100.cu), which keeps
// the error at the one-fill level for any K.
#include "gs_internal.h"

namespace gs {
namespace {

constexpr int TILE = 32;

// out[b][r][s*kp + k] (s = 0, 1, 2) from X(r, k) of batch entry b, where
// X(r, k) = X[b*stride + r*ld + k] when k_contig, else X[b*stride + k*ld + r];
// bit s of lo_mask selects the low part for segment s. Columns k in [K, kp)
// are zero. 32 x 32 tiles through shared memory keep both sides coalesced.
__global__ void __launch_bounds__(TILE * 8) k_split_tf32(const float *X, long long ld, long long stride, int rows,
                                                         int K, int kp, int k_contig, int lo_mask, int batch,
                                                         float *out, long long out_stride) {
    __shared__ float t[TILE][TILE + 1];
    grid_dep_wait();
    grid_dep_launch();
    const int k0 = blockIdx.x * TILE, r0 = blockIdx.y * TILE;
    const int tx = threadIdx.x, ty = threadIdx.y;
    for (int b = blockIdx.z; b < batch; b += gridDim.z) {
        const float *Xb = X + static_cast<size_t>(b) * stride;
        if (k_contig) {
            for (int i = ty; i < TILE; i += 8) {
                const int r = r0 + i, k = k0 + tx;
                t[i][tx] = (r < rows && k < K) ? Xb[static_cast<size_t>(r) * ld + k] : 0.0f;
            }
        } else {
            for (int i = ty; i < TILE; i += 8) {
                const int k = k0 + i, r = r0 + tx;
                t[tx][i] = (r < rows && k < K) ? Xb[static_cast<size_t>(k) * ld + r] : 0.0f;
            }
        }
        __syncthreads();
        float *ob = out + static_cast<size_t>(b) * out_stride;
        for (int i = ty; i < TILE; i += 8) {
            const int r = r0 + i, k = k0 + tx;
            if (r < rows && k < kp) {
                const float v = t[i][tx];
                const float hi = __uint_as_float(__float_as_uint(v) & 0xffffe000u);
                const float lo = v - hi;
                float *o = ob + static_cast<size_t>(r) * (3 * static_cast<size_t>(kp)) + k;
                o[0] = (lo_mask & 1) ? lo : hi;
                o[kp] = (lo_mask & 2) ? lo : hi;
                o[2 * static_cast<size_t>(kp)] = (lo_mask & 4) ? lo : hi;
            }
        }
        __syncthreads();
    }
}

cudaError_t split(Context &ctx, const float *X, long long ld, long long stride, int rows, int K, int kp, bool k_contig,
                  int lo_mask, int batch, float *out) {
    const dim3 grid((kp + TILE - 1) / TILE, (rows + TILE - 1) / TILE, batch < 65535 ? batch : 65535);
    const long long out_stride = static_cast<long long>(rows) * 3 * kp;
    const cudaError_t e = launch_pdl(k_split_tf32, grid, dim3(TILE, 8), 0, ctx.stream, 1, X, ld, stride, rows, K, kp,
                                     k_contig ? 1 : 0, lo_mask, batch, out, out_stride);
    ctx.launches++;
    return e;
}

}  // namespace

// The split costs two extra launches and 4x the operand bytes; below about a
// GFLOP, or with an output too thin for a 128-row tile, the FFMA kernel is as fast.
bool tf32_worthwhile(const GemmDesc &d) {
    const double flops = 2.0 * d.m * d.n * static_cast<double>(d.k) * d.batch;
    const long long kp = (static_cast<long long>(d.k) + 3) / 4 * 4;
    // (rows of the split grid: 32 per block, at most 65535 blocks)
    return flops >= 1.0e9 && d.m >= 128 && d.n >= 128 && 3 * kp <= 0x7fffffffLL && d.m <= 65535 * 32 &&
           d.n <= 65535 * 32;
}

cudaError_t launch_tf32(Context &ctx, const GemmDesc &d) {
    const long long kp = (static_cast<long long>(d.k) + 3) / 4 * 4;  // K' rows of 3*kp floats: 16-byte strides
    const int batch_a = (d.batch > 1 && d.stride_a != 0) ? d.batch : 1;
    const int batch_b = (d.batch > 1 && d.stride_b != 0) ? d.batch : 1;
    const size_t a_elems = static_cast<size_t>(batch_a) * d.m * 3 * kp;
    const size_t b_elems = static_cast<size_t>(batch_b) * d.n * 3 * kp;
    const size_t a_bytes = (a_elems * sizeof(float) + 255) / 256 * 256;
    const size_t need = a_bytes + b_elems * sizeof(float);
    // The split operands are 3x the f32 operands and stay allocated with the
    // handle; past 16 GiB the caller's memory matters more than the speed-up.
    if (need > (static_cast<size_t>(16) << 30)) return cudaErrorMemoryAllocation;
    if (ctx.tf32_bytes < need) {
        if (ctx.tf32_buf) cudaFree(ctx.tf32_buf);
        ctx.tf32_buf = nullptr;
        ctx.tf32_bytes = 0;
        const cudaError_t e = cudaMalloc(&ctx.tf32_buf, need);
        if (e != cudaSuccess) return e;
        ctx.tf32_bytes = need;
    }
    float *Ap = static_cast<float *>(ctx.tf32_buf);
    float *Bp = reinterpret_cast<float *>(static_cast<uint8_t *>(ctx.tf32_buf) + a_bytes);
    // A(m, k): op T stores A as k x m, so A(m, k) = A[m*lda + k] is K-contiguous.
    cudaError_t e = split(ctx, static_cast<const float *>(d.A), d.lda, d.stride_a, d.m, d.k, static_cast<int>(kp),
                          d.trans_a != 0, /*lo in segment 2*/ 4, batch_a, Ap);
    if (e != cudaSuccess) return e;
    // B(k, n): op N stores B as k x n, so B(k, n) = B[n*ldb + k] is K-contiguous.
    e = split(ctx, static_cast<const float *>(d.B), d.ldb, d.stride_b, d.n, d.k, static_cast<int>(kp), d.trans_b == 0,
              /*lo in segment 1*/ 2, batch_b, Bp);
    if (e != cudaSuccess) return e;
    GemmDesc t = d;
    t.in_kind = IN_TF32;
    t.trans_a = 1;  // A' stored K-major: 3kp x m
    t.trans_b = 0;  // B' stored K-major: 3kp x n
    t.k = static_cast<int>(3 * kp);
    t.A = Ap;
    t.lda = 3 * kp;
    t.stride_a = batch_a > 1 ? static_cast<long long>(d.m) * 3 * kp : 0;
    t.B = Bp;
    t.ldb = 3 * kp;
    t.stride_b = batch_b > 1 ? static_cast<long long>(d.n) * 3 * kp : 0;
    return launch_tc(ctx, t);
}

}  // namespace gs
