"""GPU parity of the pipelined host-buffer entry point gs_host_gemm_ex at sizes
that make it cut C into several chunks (column blocks of one GEMM, ranges of
batch entries, or — for large op N x op N GEMMs — a 4 x 4 grid of blocks fed by
alternating row blocks of A and column blocks of B) with uploads, kernels and
downloads overlapped on three streams. Checked against the oracle's exact per-element loop on sampled
entries (plus whole first/last columns) and, for INT8, exact checksums.
Bytes of C outside the matrix (padding between columns) must come back
unchanged.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import COMPUTE, OUT_OF, TOL, make_c, make_input, normwise_rel_err

pytestmark = pytest.mark.gpu


def _ext(layout, rows, cols, ld):
    return (rows - 1) * ld + cols if layout == orc.ROW_MAJOR else (cols - 1) * ld + rows


def _idx(layout, ld, r, c):
    return r * ld + c if layout == orc.ROW_MAJOR else r + c * ld


@pytest.mark.parametrize("dt,layout,op_a,op_b,m,n,k,batch,beta,ldc_pad", [
    (gs.R_8I, orc.COL_MAJOR, 0, 0, 4096, 4096, 256, 1, 0.0, 0),     # column chunks, Y uploaded per chunk
    (gs.R_16F, orc.COL_MAJOR, 0, 1, 4096, 4096, 512, 1, 0.0, 0),    # op T B: Y uploaded whole
    (gs.R_16F, orc.ROW_MAJOR, 1, 0, 2048, 4096, 512, 1, 0.5, 8),    # row-major, beta != 0, padded ldc
    (gs.R_16F, orc.COL_MAJOR, 0, 0, 512, 512, 1024, 64, 0.0, 0),    # batch-range chunks
    (gs.R_8I, orc.COL_MAJOR, 1, 0, 256, 512, 256, 96, 1.0, 0),      # batched INT8, beta != 0
    (gs.R_16F, orc.COL_MAJOR, 0, 0, 2304, 2560, 320, 1, 0.5, 8),    # 2-D blocks, beta != 0, padded ldc
    (gs.R_16BF, orc.ROW_MAJOR, 0, 0, 2048, 3072, 256, 1, 0.0, 4),   # 2-D blocks (row-major), padding kept
])
def test_pipelined_host_mirror(handle, dt, layout, op_a, op_b, m, n, k, batch, beta, ldc_pad):
    rng = np.random.default_rng(m + n + k + batch)
    ct = OUT_OF[dt]
    comp = COMPUTE[dt]
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    rm = layout == orc.ROW_MAJOR
    lda = ac if rm else ar
    ldb = bc if rm else br
    ldc = (n if rm else m) + ldc_pad
    sa, sb, sc = _ext(layout, ar, ac, lda), _ext(layout, br, bc, ldb), _ext(layout, m, n, ldc)
    a = make_input(rng, sa * batch, dt)
    b = make_input(rng, sb * batch, dt)
    c0 = make_c(rng, sc * batch, ct)
    alpha = 2.0 if dt == gs.R_8I else 1.25
    got = c0.copy()
    handle.host_gemm_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, got, ct, ldc, comp, layout=layout,
                        batch=batch)

    # padding between columns / rows comes back unchanged
    mask = np.zeros(got.size, bool)
    rows, cols = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
    for bt in range(batch):
        mask[bt * sc + _idx(layout, ldc, rows, cols).ravel()] = True
    np.testing.assert_array_equal(got[~mask], c0[~mask])

    # exact oracle values on sampled entries plus the first and last column
    cnt = 3000
    bi = np.concatenate([rng.integers(0, batch, cnt), np.zeros(m, np.int64), np.full(m, batch - 1)])
    ri = np.concatenate([rng.integers(0, m, cnt), np.arange(m), np.arange(m)])
    ci = np.concatenate([rng.integers(0, n, cnt), np.zeros(m, np.int64), np.full(m, n - 1)])
    rc, ref = orc.gemm_ex_entries((op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, c0, ct, ldc),
                                  dict(compute_type=comp, layout=layout, batch=batch, sa=sa, sb=sb, sc=sc),
                                  bi, ri, ci, got.dtype)
    assert rc == orc.OK
    sel = got[bi * sc + _idx(layout, ldc, ri, ci)]
    if ct == gs.R_32I:
        np.testing.assert_array_equal(sel, ref)
    else:
        assert normwise_rel_err(sel, ref) <= TOL[dt]
    assert handle.device_error() == 0
