"""GPU parity of gs_host_gemm_batched_ex, the host-buffer mirror of
gemm.gemmBatchedEx (src/gemm.zig:636-663): lists of host buffers, one per
entry, each at least one matrix extent long (longer buffers are allowed and
their tails stay untouched). Checked against the oracle's restatement of the
same loop: INT8 bit for bit, floats within the normwise tolerances. Also the
reference's error behaviour: differing list lengths fail before any entry is
touched; an entry whose buffer is too small fails the call after the entries
before it were computed, and leaves itself and later entries unchanged.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import COMPUTE, OUT_OF, TOL, make_c, make_input, normwise_rel_err

pytestmark = pytest.mark.gpu


def _ext(layout, rows, cols, ld):
    if rows == 0 or cols == 0:
        return 0
    return (rows - 1) * ld + cols if layout == orc.ROW_MAJOR else (cols - 1) * ld + rows


def _case(rng, dt, layout, op_a, op_b, m, n, k, count, pad, extra):
    ct = OUT_OF[dt]
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    rm = layout == orc.ROW_MAJOR
    lda = (ac if rm else ar) + pad
    ldb = (bc if rm else br) + pad
    ldc = (n if rm else m) + pad
    ea, eb, ec = _ext(layout, ar, ac, lda), _ext(layout, br, bc, ldb), _ext(layout, m, n, ldc)
    a = [make_input(rng, max(1, ea + int(rng.integers(0, extra + 1))), dt) for _ in range(count)]
    b = [make_input(rng, max(1, eb + int(rng.integers(0, extra + 1))), dt) for _ in range(count)]
    c = [make_c(rng, max(1, ec + int(rng.integers(0, extra + 1))), ct) for _ in range(count)]
    return ct, lda, ldb, ldc, a, b, c


def _check(got, ref, ct, dt):
    for g, r in zip(got, ref):
        if ct == gs.R_32I:
            np.testing.assert_array_equal(g, r)
        else:
            tol = TOL[ct] if ct in (gs.R_16F, gs.R_16BF) else TOL[dt]
            assert normwise_rel_err(g, r) <= tol


@pytest.mark.parametrize("dt,layout,op_a,op_b,m,n,k,count,beta,pad", [
    (gs.R_16F, orc.COL_MAJOR, 0, 0, 256, 384, 128, 5, 0.0, 0),
    (gs.R_16BF, orc.ROW_MAJOR, 1, 0, 200, 136, 72, 3, 0.5, 8),
    (gs.R_8I, orc.COL_MAJOR, 1, 1, 128, 256, 256, 4, 1.0, 0),
    (gs.R_8I, orc.ROW_MAJOR, 0, 1, 96, 80, 64, 2, -2.0, 16),
    (gs.R_32F, orc.COL_MAJOR, 0, 2, 130, 70, 50, 3, -1.25, 3),
    (gs.R_16F, orc.COL_MAJOR, 0, 0, 33, 17, 9, 7, 0.5, 1),     # ld not 16-byte aligned: CUDA-core path
    (gs.R_16F, orc.COL_MAJOR, 0, 0, 64, 64, 0, 2, 0.5, 0),     # k == 0: C = beta*C
])
def test_host_batched_matches_oracle(handle, dt, layout, op_a, op_b, m, n, k, count, beta, pad):
    rng = np.random.default_rng(m * 7 + n + k + count)
    comp = COMPUTE[dt]
    ct, lda, ldb, ldc, a, b, c0 = _case(rng, dt, layout, op_a, op_b, m, n, k, count, pad, extra=40)
    alpha = 2.0 if dt == gs.R_8I else 1.25
    got = [x.copy() for x in c0]
    handle.host_gemm_batched_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, got, ct, ldc, comp,
                                layout=layout)
    ref = [x.copy() for x in c0]
    assert orc.gemm_batched_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, ref, ct, ldc,
                               compute_type=comp, layout=layout) == orc.OK
    ec = _ext(layout, m, n, ldc)
    for g, c in zip(got, c0):          # tails past one extent untouched
        np.testing.assert_array_equal(g[ec:], c[ec:])
    _check(got, ref, ct, dt)
    assert handle.device_error() == 0


def test_host_batched_count_mismatch_touches_nothing(handle):
    rng = np.random.default_rng(5)
    dt = gs.R_16F
    ct, lda, ldb, ldc, a, b, c0 = _case(rng, dt, orc.COL_MAJOR, 0, 0, 64, 64, 64, 3, 0, 0)
    got = [x.copy() for x in c0]
    s = handle.host_gemm_batched_ex(0, 0, 64, 64, 64, 1.0, a, dt, lda, b[:2], dt, ldb, 0.0, got, ct, ldc,
                                    COMPUTE[dt], check=False)
    assert s == gs.STATUS_INVALID_VALUE
    assert orc.gemm_batched_ex(0, 0, 64, 64, 64, 1.0, a, dt, lda, b[:2], dt, ldb, 0.0, [x.copy() for x in c0], ct,
                               ldc) == orc.ERR_INVALID_BATCH_COUNT
    for g, c in zip(got, c0):
        np.testing.assert_array_equal(g, c)


@pytest.mark.parametrize("bad", [0, 2, 4])
def test_host_batched_short_entry_keeps_prefix(handle, bad):
    rng = np.random.default_rng(11 + bad)
    dt, m, n, k, count = gs.R_8I, 128, 96, 64, 5
    ct, lda, ldb, ldc, a, b, c0 = _case(rng, dt, orc.COL_MAJOR, 0, 0, m, n, k, count, 0, 0)
    b[bad] = b[bad][:-1]                                  # one element short: BufferTooSmall
    got = [x.copy() for x in c0]
    s = handle.host_gemm_batched_ex(0, 0, m, n, k, 3.0, a, dt, lda, b, dt, ldb, 1.0, got, ct, ldc, COMPUTE[dt],
                                    check=False)
    assert s == gs.STATUS_INVALID_VALUE
    assert "entry %d" % bad in handle.last_error()
    ref = [x.copy() for x in c0]
    assert orc.gemm_batched_ex(0, 0, m, n, k, 3.0, a, dt, lda, b, dt, ldb, 1.0, ref, ct, ldc,
                               compute_type=COMPUTE[dt]) == orc.ERR_BUFFER_TOO_SMALL
    for j in range(count):
        np.testing.assert_array_equal(got[j], ref[j])     # prefix computed, the rest unchanged
        if j >= bad:
            np.testing.assert_array_equal(got[j], c0[j])
    assert handle.device_error() == 0


def test_host_batched_empty_lists(handle):
    assert handle.host_gemm_batched_ex(0, 0, 8, 8, 8, 1.0, [], gs.R_16F, 8, [], gs.R_16F, 8, 0.0, [], gs.R_32F, 8,
                                       gs.COMPUTE_32F, check=False) == gs.STATUS_SUCCESS


def test_host_gemm_ex_k0_ignores_leading_dimensions(handle):
    """src/gemm.zig checks no leading dimension; with k == 0 nothing but C is touched, so ld 0 is accepted."""
    rng = np.random.default_rng(3)
    m, n = 64, 48
    a = make_input(rng, 1, gs.R_16F)
    b = make_input(rng, 1, gs.R_16F)
    c0 = make_c(rng, m * n, gs.R_32F)
    got = c0.copy()
    handle.host_gemm_ex(0, 0, m, n, 0, 2.0, a, gs.R_16F, 0, b, gs.R_16F, 0, 0.5, got, gs.R_32F, m, gs.COMPUTE_32F)
    ref = c0.copy()
    assert orc.gemm_ex(0, 0, m, n, 0, 2.0, a, gs.R_16F, 0, b, gs.R_16F, 0, 0.5, ref, gs.R_32F, m,
                       compute_type=gs.COMPUTE_32F) == orc.OK
    np.testing.assert_array_equal(got, ref)
