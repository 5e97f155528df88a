// host_mirror.cu -- gs_host_gemm_ex: the host-buffer counterpart of
// slang-gemm's gemm.gemmEx / gemm.gemmStridedBatchedEx (src/gemm.zig:546-576,
// :632-634, :671-706). It takes the same ExDesc fields (host byte slices with
// lengths, row- or column-major layout, stride 0 = one matrix extent),
// validates them like validateByteSliceLen (src/gemm.zig:769-775), stages the
// operands in device memory owned by the handle and runs the device path.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "gs_internal.h"

namespace {

size_t type_size(int t) {
    switch (t) {
    case GS_R_16F: case GS_R_16BF: return 2;
    case GS_R_32F: case GS_R_32I: return 4;
    case GS_R_8I: return 1;
    case GS_R_64F: return 8;
    default: return 0;
    }
}

// matrixExtent with matrixLayout(layout, ld) (src/gemm.zig:165-170, :708-711).
size_t extent(int layout, size_t ld, size_t rows, size_t cols) {
    if (rows == 0 || cols == 0) return 0;
    if (layout == GS_LAYOUT_ROW_MAJOR) return (rows - 1) * ld + (cols - 1) + 1;
    return (rows - 1) + (cols - 1) * ld + 1;
}

// m, n and k the device entry points accept (their kernels' tile coordinates
// are 32-bit); checked here before anything is staged.
constexpr size_t kMaxDim = 0x7fffffff - 1024;

// validateByteSliceLen (src/gemm.zig:769-775); `stride` already resolved.
gs_status check_len(size_t len, size_t es, size_t ext, size_t stride, size_t batch, const char *what, std::string *why) {
    if (ext == 0) return GS_STATUS_SUCCESS;
    if (stride < ext) {
        *why = std::string(what) + ": stride smaller than one matrix extent (InvalidStride)";
        return GS_STATUS_INVALID_VALUE;
    }
    const size_t need = ((batch - 1) * stride + ext) * es;
    if (len < need) {
        *why = std::string(what) + ": buffer too small (BufferTooSmall)";
        return GS_STATUS_INVALID_VALUE;
    }
    return GS_STATUS_SUCCESS;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// f32 -> f16 bits, round to nearest even (finite, normal-range values; alpha/beta of COMPUTE_16F).
uint16_t f32_to_f16_rne(float v) {
    uint32_t x;
    std::memcpy(&x, &v, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int e = static_cast<int>((x >> 23) & 0xffu) - 127 + 15;
    const uint32_t man = x & 0x7fffffu;
    if (v == 0.0f) return static_cast<uint16_t>(sign);
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    if (e <= 0) return static_cast<uint16_t>(sign);
    uint32_t val = (static_cast<uint32_t>(e) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (val & 1u))) val++;
    return static_cast<uint16_t>(sign | val);
}

// alpha / beta in the compute type's host representation: float for 32F*,
// int32 for 32I* (integral values only), f16 bits for 16F*.
struct HostScalars {
    float f[2];
    int32_t i[2];
    uint16_t h[2];
    const void *alpha = nullptr, *beta = nullptr;
    bool set(int compute, double a, double b) {
        f[0] = static_cast<float>(a);
        f[1] = static_cast<float>(b);
        alpha = &f[0];
        beta = &f[1];
        if (compute == GS_COMPUTE_32I || compute == GS_COMPUTE_32I_PEDANTIC) {
            if (a != std::floor(a) || b != std::floor(b) || std::fabs(a) > 2147483647.0 || std::fabs(b) > 2147483647.0)
                return false;
            i[0] = static_cast<int32_t>(a);
            i[1] = static_cast<int32_t>(b);
            alpha = &i[0];
            beta = &i[1];
        } else if (compute == GS_COMPUTE_16F || compute == GS_COMPUTE_16F_PEDANTIC) {
            h[0] = f32_to_f16_rne(f[0]);
            h[1] = f32_to_f16_rne(f[1]);
            alpha = &h[0];
            beta = &h[1];
        }
        return true;
    }
};

}  // namespace

extern "C" gs_status gs_gemm_strided_batched_ex(gs_handle, int, int, int, int, int, const void *, const void *, int,
                                                int, long long, const void *, int, int, long long, const void *, void *,
                                                int, int, long long, int, int, int);


extern "C" gs_status gs_host_gemm_ex(gs_handle h, const gs_ex_desc *d) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    gs::Context &ctx = h->ctx;
    if (!d) return GS_STATUS_INVALID_VALUE;
    std::string why;
    if (d->batch_count == 0) {
        ctx.last_error = "batch_count == 0 (InvalidBatchCount)";
        return GS_STATUS_INVALID_VALUE;
    }
    if (d->layout != GS_LAYOUT_ROW_MAJOR && d->layout != GS_LAYOUT_COL_MAJOR) {
        ctx.last_error = "invalid layout";
        return GS_STATUS_INVALID_VALUE;
    }
    const size_t esa = type_size(d->a_type), esb = type_size(d->b_type), esc = type_size(d->c_type);
    if (!esa || !esb || !esc) {
        ctx.last_error = "unsupported data type";
        return GS_STATUS_NOT_SUPPORTED;
    }
    const bool ta = d->op_a != GS_OP_N, tb = d->op_b != GS_OP_N;
    const size_t a_ext = extent(d->layout, d->lda, ta ? d->k : d->m, ta ? d->m : d->k);
    const size_t b_ext = extent(d->layout, d->ldb, tb ? d->n : d->k, tb ? d->k : d->n);
    const size_t c_ext = extent(d->layout, d->ldc, d->m, d->n);
    const size_t sa = d->stride_a ? d->stride_a : a_ext;
    const size_t sb = d->stride_b ? d->stride_b : b_ext;
    const size_t sc = d->stride_c ? d->stride_c : c_ext;
    gs_status st;
    if ((st = check_len(d->a_len, esa, a_ext, sa, d->batch_count, "a", &why)) != GS_STATUS_SUCCESS ||
        (st = check_len(d->b_len, esb, b_ext, sb, d->batch_count, "b", &why)) != GS_STATUS_SUCCESS ||
        (st = check_len(d->c_len, esc, c_ext, sc, d->batch_count, "c", &why)) != GS_STATUS_SUCCESS) {
        ctx.last_error = why;
        return st;
    }
    if (d->m == 0 || d->n == 0) return GS_STATUS_SUCCESS;
    const size_t lim = 0x7fffffff;
    if (d->m > kMaxDim || d->n > kMaxDim || d->k > kMaxDim || d->lda > lim || d->ldb > lim || d->ldc > lim ||
        d->batch_count > lim) {
        ctx.last_error = "dimension exceeds the 32-bit device API";
        return GS_STATUS_NOT_SUPPORTED;
    }

    HostScalars sc_ab;
    if (!sc_ab.set(d->compute_type, d->alpha_re, d->beta_re)) {
        ctx.last_error = "32I compute needs integral alpha/beta";
        return GS_STATUS_NOT_SUPPORTED;
    }
    const void *alpha = sc_ab.alpha, *beta = sc_ab.beta;

    // Stage A, B, C in one device region.
    const size_t a_bytes = ((d->batch_count - 1) * sa + a_ext) * esa;
    const size_t b_bytes = ((d->batch_count - 1) * sb + b_ext) * esb;
    const size_t c_bytes = ((d->batch_count - 1) * sc + c_ext) * esc;
    const size_t off_b = round_up(a_bytes, 256), off_c = off_b + round_up(b_bytes, 256);
    const size_t need = off_c + round_up(c_bytes, 256);
    if (ctx.stage_bytes < need) {
        if (ctx.stage) cudaFree(ctx.stage);
        ctx.stage = nullptr;
        ctx.stage_bytes = 0;
        if (cudaMalloc(&ctx.stage, need) != cudaSuccess) {
            cudaGetLastError();
            ctx.last_error = "device staging allocation failed";
            return GS_STATUS_ALLOC_FAILED;
        }
        ctx.stage_bytes = need;
    }
    uint8_t *dA = static_cast<uint8_t *>(ctx.stage);
    uint8_t *dB = dA + off_b;
    uint8_t *dC = dA + off_c;
    // C is uploaded whenever it is read (beta != 0) or has bytes between its
    // elements that the download must leave untouched.
    const bool c_dense = (d->layout == GS_LAYOUT_COL_MAJOR ? d->ldc == d->m : d->ldc == d->n) &&
                         (d->batch_count == 1 || sc == c_ext);
    const bool upload_c = d->beta_re != 0.0 || !c_dense;

    // Row-major C = op(A) op(B) is column-major C^T = op(B)^T op(A)^T: X, Y are
    // the column-major operands of that problem, C' its column-major result.
    const bool rm = d->layout == GS_LAYOUT_ROW_MAJOR;
    const int m = static_cast<int>(rm ? d->n : d->m), n = static_cast<int>(rm ? d->m : d->n);
    const int opx = rm ? d->op_b : d->op_a, opy = rm ? d->op_a : d->op_b;
    uint8_t *dX = rm ? dB : dA, *dY = rm ? dA : dB;
    const uint8_t *hX = static_cast<const uint8_t *>(rm ? d->b : d->a);
    const uint8_t *hY = static_cast<const uint8_t *>(rm ? d->a : d->b);
    const size_t esx = rm ? esb : esa, esy = rm ? esa : esb;
    const size_t ext_x = rm ? b_ext : a_ext, ext_y = rm ? a_ext : b_ext;
    const int ldx = static_cast<int>(rm ? d->ldb : d->lda), ldy = static_cast<int>(rm ? d->lda : d->ldb);
    // src/gemm.zig never checks a leading dimension, and with k == 0 neither
    // operand is read: any ld the device API accepts will do there.
    const int ld_k0 = static_cast<int>(std::max<size_t>({1, d->m, d->n}));
    const int ldx_dev = d->k == 0 ? ld_k0 : ldx, ldy_dev = d->k == 0 ? ld_k0 : ldy;
    const size_t sx = rm ? sb : sa, sy = rm ? sa : sb;
    const int tx = rm ? d->b_type : d->a_type, ty = rm ? d->a_type : d->b_type;
    const size_t batch = d->batch_count;

    // Pipeline: stream h2d uploads, the handle's stream computes, stream d2h
    // downloads. C' is cut into chunks (column blocks of one GEMM, or ranges of
    // batch entries); each chunk's kernel waits for its uploads and its
    // download waits for its kernel, so copies in both directions overlap each
    // other and the tensor cores.
    cudaError_t e = cudaSuccess;
    if (!ctx.h2d) {
        e = cudaStreamCreateWithFlags(&ctx.h2d, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx.d2h, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx.ev_start, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx.ev_a, cudaEventDisableTiming);
        for (int i = 0; e == cudaSuccess && i < gs::Context::kMaxChunks; ++i) {
            e = cudaEventCreateWithFlags(&ctx.ev_in[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx.ev_out[i], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) {
            ctx.last_error = std::string("pipeline streams/events: ") + cudaGetErrorString(e);
            return GS_STATUS_EXECUTION_FAILED;
        }
    }
    const size_t units = batch > 1 ? batch : static_cast<size_t>(n);
    const size_t align = batch > 1 ? 1 : 256;
    const size_t total_bytes = a_bytes + b_bytes + c_bytes * (upload_c ? 2 : 1);
    size_t chunks = total_bytes / (32u << 20);
    chunks = std::max<size_t>(1, std::min<size_t>({chunks, static_cast<size_t>(16), (units + align - 1) / align}));
    // Only a contiguous Y column block can be uploaded per chunk (op N); otherwise Y goes first, whole.
    const bool y_chunked = batch == 1 && opy == GS_OP_N;
    cudaStream_t s = ctx.stream;
    auto h2d = [&](uint8_t *dst, const uint8_t *src, size_t bytes) {
        if (e == cudaSuccess && bytes > 0) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx.h2d);
    };
    if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_start, s);  // work already queued on the handle's stream
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx.h2d, ctx.ev_start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx.d2h, ctx.ev_start, 0);

    // Large single GEMM with X and Y both op N: 2-D pipeline. The first block
    // of C needs only one row block of X and one column block of Y, instead of
    // all of X, so downloads start after 1/R + 1/Q of the operand bytes. X row
    // blocks and Y column blocks are uploaded alternately; after each upload
    // the C blocks it completes are computed and downloaded (pitched copies).
    const int RB = 4, QB = 4;
    const bool two_d = batch == 1 && opx == GS_OP_N && opy == GS_OP_N && m >= 2048 && n >= 2048 && d->k >= 256 &&
                       e == cudaSuccess;
    if (two_d) {
        size_t rcut[RB + 1], qcut[QB + 1];
        for (int i = 0; i <= RB; ++i) rcut[i] = i == RB ? static_cast<size_t>(m) : (static_cast<size_t>(m) * i / RB) / 256 * 256;
        for (int j = 0; j <= QB; ++j) qcut[j] = j == QB ? static_cast<size_t>(n) : (static_cast<size_t>(n) * j / QB) / 256 * 256;
        const size_t ldxb = static_cast<size_t>(ldx) * esx, ldyb = static_cast<size_t>(ldy) * esy;
        const size_t ldcb = d->ldc * esc;
        int ev_n = 0;  // upload events used
        int rows_up = 0, cols_up = 0;
        auto issue_block = [&](int i, int j, cudaEvent_t ready) {
            const size_t r0 = rcut[i], r1 = rcut[i + 1], c0 = qcut[j], c1 = qcut[j + 1];
            const size_t coff = r0 * esc + c0 * ldcb;
            cudaEvent_t in = ready;
            // Only the block's own rows are written back, so padding between columns never
            // needs the upload: C is uploaded only when it is read.
            if (d->beta_re != 0.0 && e == cudaSuccess) {
                e = cudaMemcpy2DAsync(dC + coff, ldcb, static_cast<const uint8_t *>(d->c) + coff, ldcb,
                                      (r1 - r0) * esc, c1 - c0, cudaMemcpyHostToDevice, ctx.h2d);
                if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_in[ev_n], ctx.h2d);
                in = ctx.ev_in[ev_n++];
            }
            if (e == cudaSuccess) e = cudaStreamWaitEvent(s, in, 0);
            if (e != cudaSuccess) return;
            st = gs_gemm_strided_batched_ex(h, GS_OP_N, GS_OP_N, static_cast<int>(r1 - r0), static_cast<int>(c1 - c0),
                                            static_cast<int>(d->k), alpha, dX + r0 * esx, tx, ldx, 0,
                                            dY + c0 * ldyb, ty, ldy, 0, beta, dC + coff, d->c_type,
                                            static_cast<int>(d->ldc), 0, 1, d->compute_type, d->algo);
            if (st != GS_STATUS_SUCCESS) return;
            const int blk = i * QB + j;
            e = cudaEventRecord(ctx.ev_out[blk], s);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx.d2h, ctx.ev_out[blk], 0);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(static_cast<uint8_t *>(d->c) + coff, ldcb, dC + coff, ldcb, (r1 - r0) * esc,
                                      c1 - c0, cudaMemcpyDeviceToHost, ctx.d2h);
        };
        for (int step = 0; step < RB + QB && e == cudaSuccess && st == GS_STATUS_SUCCESS; ++step) {
            const bool take_row = (step % 2 == 0 && rows_up < RB) || cols_up == QB;
            if (take_row) {
                const size_t r0 = rcut[rows_up], r1 = rcut[rows_up + 1];
                e = cudaMemcpy2DAsync(dX + r0 * esx, ldxb, hX + r0 * esx, ldxb, (r1 - r0) * esx, d->k,
                                      cudaMemcpyHostToDevice, ctx.h2d);
                if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_in[ev_n], ctx.h2d);
                cudaEvent_t ready = ctx.ev_in[ev_n++];
                for (int j = 0; j < cols_up && e == cudaSuccess && st == GS_STATUS_SUCCESS; ++j)
                    issue_block(rows_up, j, ready);
                ++rows_up;
            } else {
                const size_t c0 = qcut[cols_up], c1 = qcut[cols_up + 1];
                const size_t y0 = c0 * ldyb, y1 = ((c1 - 1) * ldy + d->k) * esy;
                e = cudaMemcpyAsync(dY + y0, hY + y0, y1 - y0, cudaMemcpyHostToDevice, ctx.h2d);
                if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_in[ev_n], ctx.h2d);
                cudaEvent_t ready = ctx.ev_in[ev_n++];
                for (int i = 0; i < rows_up && e == cudaSuccess && st == GS_STATUS_SUCCESS; ++i)
                    issue_block(i, cols_up, ready);
                ++cols_up;
            }
        }
        if (st != GS_STATUS_SUCCESS) {
            cudaStreamSynchronize(ctx.h2d);
            cudaStreamSynchronize(ctx.d2h);
            return st;
        }
    }
    if (!two_d && batch == 1) {
        h2d(dX, hX, ext_x * esx);
        if (!y_chunked) h2d(dY, hY, ext_y * esy);
        if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_a, ctx.h2d);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ctx.ev_a, 0);
    }
    for (size_t j = 0; !two_d && j < chunks && e == cudaSuccess; ++j) {
        size_t u0 = units * j / chunks, u1 = units * (j + 1) / chunks;
        if (j > 0) u0 = (u0 / align) * align;
        if (j + 1 < chunks) u1 = (u1 / align) * align;
        if (u1 <= u0) continue;
        size_t c0, c1;  // byte range of C' this chunk covers
        const uint8_t *X = dX, *Y = dY;
        uint8_t *C = dC;
        int nn = n, bb = static_cast<int>(batch);
        if (batch == 1) {
            c0 = u0 * d->ldc * esc;
            c1 = ((u1 - 1) * d->ldc + static_cast<size_t>(m)) * esc;
            if (y_chunked) {
                const size_t y0 = u0 * ldy * esy, y1 = ext_y == 0 ? y0 : ((u1 - 1) * ldy + d->k) * esy;
                h2d(dY + y0, hY + y0, y1 - y0);
                Y = dY + y0;
            } else {
                Y = dY + u0 * esy;  // op T: column j of C' reads row j of the stored (n' x k) Y
            }
            C = dC + c0;
            nn = static_cast<int>(u1 - u0);
        } else {
            const size_t x0 = u0 * sx * esx, x1 = ((u1 - 1) * sx + ext_x) * esx;
            const size_t y0 = u0 * sy * esy, y1 = ((u1 - 1) * sy + ext_y) * esy;
            if (ext_x) h2d(dX + x0, hX + x0, x1 - x0);
            if (ext_y) h2d(dY + y0, hY + y0, y1 - y0);
            c0 = u0 * sc * esc;
            c1 = ((u1 - 1) * sc + c_ext) * esc;
            X = dX + x0;
            Y = dY + y0;
            C = dC + c0;
            bb = static_cast<int>(u1 - u0);
        }
        if (upload_c) h2d(dC + c0, static_cast<const uint8_t *>(d->c) + c0, c1 - c0);
        if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_in[j], ctx.h2d);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ctx.ev_in[j], 0);
        if (e != cudaSuccess) break;
        st = gs_gemm_strided_batched_ex(h, opx, opy, m, nn, static_cast<int>(d->k), alpha, X, tx, ldx_dev,
                                        static_cast<long long>(sx), Y, ty, ldy_dev, static_cast<long long>(sy), beta, C,
                                        d->c_type, static_cast<int>(d->ldc), static_cast<long long>(sc), bb,
                                        d->compute_type, d->algo);
        if (st != GS_STATUS_SUCCESS) {
            cudaStreamSynchronize(ctx.h2d);
            return st;
        }
        e = cudaEventRecord(ctx.ev_out[j], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx.d2h, ctx.ev_out[j], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<uint8_t *>(d->c) + c0, dC + c0, c1 - c0, cudaMemcpyDeviceToHost, ctx.d2h);
    }
    // Leave the handle's stream ordered after the downloads, then wait for all of it.
    if (e == cudaSuccess) e = cudaEventRecord(ctx.ev_start, ctx.d2h);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ctx.ev_start, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cudaStreamSynchronize(ctx.h2d);
        cudaStreamSynchronize(ctx.d2h);
        ctx.last_error = std::string("host-buffer pipeline: ") + cudaGetErrorString(e);
        return GS_STATUS_EXECUTION_FAILED;
    }
    return GS_STATUS_SUCCESS;
}

// gemm.gemmBatchedEx over host buffers (src/gemm.zig:636-663). Each entry is an
// ExDesc with batch_count 1 (stride = one extent); the valid prefix of entries
// is packed into the staging region at extent strides and computed by one
// strided-batched call.
extern "C" gs_status gs_host_gemm_batched_ex(gs_handle h, const gs_ptr_batched_desc *d) {
    if (!h) return GS_STATUS_NOT_INITIALIZED;
    gs::Context &ctx = h->ctx;
    if (!d) return GS_STATUS_INVALID_VALUE;
    if (d->a_count != d->b_count || d->a_count != d->c_count) {
        ctx.last_error = "pointer counts differ (InvalidBatchCount)";
        return GS_STATUS_INVALID_VALUE;
    }
    const size_t count = d->a_count;
    if (count == 0) return GS_STATUS_SUCCESS;
    if (!d->a || !d->b || !d->c || !d->a_lens || !d->b_lens || !d->c_lens) {
        ctx.last_error = "null pointer array";
        return GS_STATUS_INVALID_VALUE;
    }
    if (d->layout != GS_LAYOUT_ROW_MAJOR && d->layout != GS_LAYOUT_COL_MAJOR) {
        ctx.last_error = "invalid layout";
        return GS_STATUS_INVALID_VALUE;
    }
    const size_t esa = type_size(d->a_type), esb = type_size(d->b_type), esc = type_size(d->c_type);
    if (!esa || !esb || !esc) {
        ctx.last_error = "unsupported data type";
        return GS_STATUS_NOT_SUPPORTED;
    }
    const bool ta = d->op_a != GS_OP_N, tb = d->op_b != GS_OP_N;
    const size_t a_ext = extent(d->layout, d->lda, ta ? d->k : d->m, ta ? d->m : d->k);
    const size_t b_ext = extent(d->layout, d->ldb, tb ? d->n : d->k, tb ? d->k : d->n);
    const size_t c_ext = extent(d->layout, d->ldc, d->m, d->n);
    // The reference validates entry by entry inside its loop: find the valid prefix.
    size_t valid = 0;
    std::string why;
    gs_status bad = GS_STATUS_SUCCESS;
    for (; valid < count; ++valid) {
        std::string w;
        gs_status st;
        if ((st = check_len(d->a_lens[valid], esa, a_ext, a_ext, 1, "a", &w)) != GS_STATUS_SUCCESS ||
            (st = check_len(d->b_lens[valid], esb, b_ext, b_ext, 1, "b", &w)) != GS_STATUS_SUCCESS ||
            (st = check_len(d->c_lens[valid], esc, c_ext, c_ext, 1, "c", &w)) != GS_STATUS_SUCCESS) {
            bad = st;
            why = "entry " + std::to_string(valid) + ": " + w;
            break;
        }
    }
    gs_status st = GS_STATUS_SUCCESS;
    if (valid > 0 && d->m != 0 && d->n != 0) {
        const size_t lim = 0x7fffffff;
        if (d->m > kMaxDim || d->n > kMaxDim || d->k > kMaxDim || d->lda > lim || d->ldb > lim || d->ldc > lim ||
            valid > lim) {
            ctx.last_error = "dimension exceeds the 32-bit device API";
            return GS_STATUS_NOT_SUPPORTED;
        }
        HostScalars sc_ab;
        if (!sc_ab.set(d->compute_type, d->alpha_re, d->beta_re)) {
            ctx.last_error = "32I compute needs integral alpha/beta";
            return GS_STATUS_NOT_SUPPORTED;
        }
        // Packed staging: entry j of A at j * a_ext elements, and so on.
        const size_t a_bytes = valid * a_ext * esa, b_bytes = valid * b_ext * esb, c_bytes = valid * c_ext * esc;
        const size_t off_b = round_up(a_bytes, 256), off_c = off_b + round_up(b_bytes, 256);
        const size_t need = off_c + round_up(c_bytes, 256);
        if (ctx.stage_bytes < need) {
            if (ctx.stage) cudaFree(ctx.stage);
            ctx.stage = nullptr;
            ctx.stage_bytes = 0;
            if (cudaMalloc(&ctx.stage, need) != cudaSuccess) {
                cudaGetLastError();
                ctx.last_error = "device staging allocation failed";
                return GS_STATUS_ALLOC_FAILED;
            }
            ctx.stage_bytes = need;
        }
        uint8_t *dA = static_cast<uint8_t *>(ctx.stage), *dB = dA + off_b, *dC = dA + off_c;
        // C is uploaded when it is read, or when padding between its columns
        // (rows) would otherwise come back from the device as garbage.
        const bool c_dense = d->layout == GS_LAYOUT_COL_MAJOR ? d->ldc == d->m : d->ldc == d->n;
        const bool upload_c = d->beta_re != 0.0 || !c_dense;
        cudaStream_t s = ctx.stream;
        cudaError_t e = cudaSuccess;
        for (size_t j = 0; j < valid && e == cudaSuccess; ++j) {
            if (a_ext) e = cudaMemcpyAsync(dA + j * a_ext * esa, d->a[j], a_ext * esa, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess && b_ext)
                e = cudaMemcpyAsync(dB + j * b_ext * esb, d->b[j], b_ext * esb, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess && upload_c && c_ext)
                e = cudaMemcpyAsync(dC + j * c_ext * esc, d->c[j], c_ext * esc, cudaMemcpyHostToDevice, s);
        }
        if (e != cudaSuccess) {
            cudaStreamSynchronize(s);
            ctx.last_error = std::string("host-buffer upload: ") + cudaGetErrorString(e);
            return GS_STATUS_EXECUTION_FAILED;
        }
        const bool rm = d->layout == GS_LAYOUT_ROW_MAJOR;
        const int m = static_cast<int>(rm ? d->n : d->m), n = static_cast<int>(rm ? d->m : d->n);
        // With k == 0 neither operand is read (and src/gemm.zig checks no leading dimension).
        const size_t ld_k0 = std::max<size_t>({1, d->m, d->n});
        const size_t lda_dev = d->k == 0 ? ld_k0 : d->lda, ldb_dev = d->k == 0 ? ld_k0 : d->ldb;
        st = gs_gemm_strided_batched_ex(h, rm ? d->op_b : d->op_a, rm ? d->op_a : d->op_b, m, n, static_cast<int>(d->k),
                                        sc_ab.alpha, rm ? dB : dA, rm ? d->b_type : d->a_type,
                                        static_cast<int>(rm ? ldb_dev : lda_dev),
                                        static_cast<long long>(rm ? b_ext : a_ext), rm ? dA : dB,
                                        rm ? d->a_type : d->b_type, static_cast<int>(rm ? lda_dev : ldb_dev),
                                        static_cast<long long>(rm ? a_ext : b_ext), sc_ab.beta, dC, d->c_type,
                                        static_cast<int>(d->ldc), static_cast<long long>(c_ext),
                                        static_cast<int>(valid), d->compute_type, d->algo);
        if (st == GS_STATUS_SUCCESS) {
            for (size_t j = 0; j < valid && e == cudaSuccess; ++j)
                if (c_ext) e = cudaMemcpyAsync(d->c[j], dC + j * c_ext * esc, c_ext * esc, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                ctx.last_error = std::string("host-buffer download: ") + cudaGetErrorString(e);
                return GS_STATUS_EXECUTION_FAILED;
            }
        } else {
            cudaStreamSynchronize(s);
            return st;
        }
    }
    if (bad != GS_STATUS_SUCCESS) {
        ctx.last_error = why;
        return bad;
    }
    return st;
}
