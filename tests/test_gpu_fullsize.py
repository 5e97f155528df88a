"""Full-size parity for the north star's configurations C3, C4, C5 and C5b.

At 8192^3 the scalar oracle would need ~5e11 multiply-adds, so parity is
established through size-independent properties on the same seeded inputs:
  * exact oracle values of >= 4096 random entries plus the complete first and
    last row and column of C (or_gemm_ex_entries runs src/gemm.zig's
    per-element loop for just those entries);
  * checksums of checksums: the column sums of C equal (1^T A) B and the row
    sums equal A (B 1). For INT8 -> INT32 both are exact in int64 and must
    match bit for bit; for floats they are compared in f64 within the
    configuration's normwise tolerance.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import TOL, normwise_rel_err, to_dev

pytestmark = pytest.mark.gpu


def col_major_2d(x: np.ndarray, rows: int, cols: int, batch: int = 1) -> np.ndarray:
    """(batch, rows, cols) view of a packed column-major buffer."""
    return x.reshape(batch, cols, rows).transpose(0, 2, 1)


def sampled_entries(m: int, n: int, batch: int, rng, count: int = 4096):
    b = rng.integers(0, batch, count)
    r = rng.integers(0, m, count)
    c = rng.integers(0, n, count)
    edges_r = np.concatenate([np.zeros(n, np.int64), np.full(n, m - 1), np.arange(m), np.arange(m)])
    edges_c = np.concatenate([np.arange(n), np.arange(n), np.zeros(m, np.int64), np.full(m, n - 1)])
    edges_b = np.concatenate([np.zeros(2 * n + 2 * m, np.int64)])
    edges_b[: n + m] = 0
    edges_b[n + m:] = batch - 1
    return (np.concatenate([b, edges_b]), np.concatenate([r, edges_r]), np.concatenate([c, edges_c]))


def check(dt, ct, op_a, op_b, m, n, k, batch=1, alpha=1.0, seed=0):
    rng = np.random.default_rng(seed)
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    if dt == gs.R_8I:
        a = rng.integers(-128, 128, ar * ac * batch, dtype=np.int64).astype(np.int8)
        b = rng.integers(-128, 128, br * bc * batch, dtype=np.int64).astype(np.int8)
        c0 = np.zeros(m * n * batch, np.int32)
        comp = gs.COMPUTE_32I
    else:
        a = orc.randn_lowp(rng, ar * ac * batch, dt)
        b = orc.randn_lowp(rng, br * bc * batch, dt)
        c0 = np.zeros(m * n * batch, np.float32)
        comp = gs.COMPUTE_32F
    dc = to_dev(c0)
    with gs.Handle() as h:
        if batch == 1:
            h.gemm_ex(op_a, op_b, m, n, k, alpha, to_dev(a), dt, ar, to_dev(b), dt, br, 0.0, dc, ct, m, comp)
        else:
            h.gemm_strided_batched_ex(op_a, op_b, m, n, k, alpha, to_dev(a), dt, ar, ar * ac, to_dev(b), dt, br,
                                      br * bc, 0.0, dc, ct, m, m * n, batch, comp)
        tc = {gs.R_16F: gs.KERNEL_TC_F16, gs.R_16BF: gs.KERNEL_TC_BF16, gs.R_8I: gs.KERNEL_TC_I8}[dt]
        assert h.last_kernels() & tc
        assert h.device_error() == 0
    got = dc.cpu().numpy()

    # 1) exact oracle entries
    bi, ri, ci = sampled_entries(m, n, batch, rng)
    rc, ref = orc.gemm_ex_entries((op_a, op_b, m, n, k, alpha, a, dt, ar, b, dt, br, 0.0, c0, ct, m),
                                  dict(compute_type=comp, batch=batch, sa=ar * ac, sb=br * bc, sc=m * n),
                                  bi, ri, ci, got.dtype)
    assert rc == orc.OK
    sel = got[bi * m * n + ci * m + ri]
    if dt == gs.R_8I:
        np.testing.assert_array_equal(sel, ref)
    else:
        err = normwise_rel_err(sel, ref)
        assert err <= TOL[dt], f"sampled normwise error {err:.2e}"

    # 2) checksums of checksums
    if dt == gs.R_8I:
        A = col_major_2d(a.astype(np.int64), ar, ac, batch)
        B = col_major_2d(b.astype(np.int64), br, bc, batch)
        C = col_major_2d(got.astype(np.int64), m, n, batch)
    else:
        A = col_major_2d(orc.decode_lowp(a, dt).astype(np.float64), ar, ac, batch)
        B = col_major_2d(orc.decode_lowp(b, dt).astype(np.float64), br, bc, batch)
        C = col_major_2d(got.astype(np.float64), m, n, batch)
    if op_a != 0:
        A = A.transpose(0, 2, 1)
    if op_b != 0:
        B = B.transpose(0, 2, 1)
    for bt in range(batch):
        col_ref = (A[bt].sum(axis=0) @ B[bt]) * alpha
        row_ref = (A[bt] @ B[bt].sum(axis=1)) * alpha
        col_got = C[bt].sum(axis=0)
        row_got = C[bt].sum(axis=1)
        if dt == gs.R_8I:
            np.testing.assert_array_equal(col_got, col_ref.astype(np.int64))
            np.testing.assert_array_equal(row_got, row_ref.astype(np.int64))
        else:
            assert normwise_rel_err(col_got, col_ref) <= TOL[dt]
            assert normwise_rel_err(row_got, row_ref) <= TOL[dt]


@pytest.mark.parametrize("dt,op_a", [(gs.R_16F, 0), (gs.R_16F, 1), (gs.R_16BF, 0)])
@pytest.mark.parametrize("size", [4096, 8192])
def test_config3_gemm_ex_fullsize(dt, op_a, size):
    check(dt, gs.R_32F, op_a, 0, size, size, size, seed=size + op_a + dt)


def test_config5_int8_8192_bit_exact():
    check(gs.R_8I, gs.R_32I, 0, 0, 8192, 8192, 8192, seed=5)


def test_config4_strided_batch256():
    check(gs.R_16F, gs.R_32F, 0, 0, 512, 512, 1024, batch=256, alpha=1.0 / 32.0, seed=4)


def test_config5b_int8_strided_batch64_bit_exact():
    check(gs.R_8I, gs.R_32I, 0, 0, 2048, 2048, 2048, batch=64, seed=55)
