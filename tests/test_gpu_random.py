"""Seeded random sweep of the device entry points against the oracle.

Each case draws a data type (and output type), the two ops (N / T / C), ragged
M, N, K (K = 0 included), leading-dimension padding that is sometimes not a
multiple of 16 bytes (exercising the CUDA-core fallback), a batch of 1-3 with
padded strides, strided or pointer-array batching, alpha / beta and the tile
hint. The same bytes go through the C ABI on the GPU and through the oracle's
restatement of src/gemm.zig; INT8 must match bit for bit, floats within the
normwise tolerances, and bytes of C outside the matrices must be unchanged.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import (NP_OF, assert_parity, make_c, make_input, to_dev, to_host)

pytestmark = pytest.mark.gpu

N_CASES = 256
OUTS = {gs.R_16F: [gs.R_32F, gs.R_32F, gs.R_16F], gs.R_16BF: [gs.R_32F, gs.R_32F, gs.R_16BF], gs.R_8I: [gs.R_32I],
        gs.R_32F: [gs.R_32F]}
COMPUTES = {(gs.R_16F, gs.R_32F): [gs.COMPUTE_32F, gs.COMPUTE_32F_FAST_16F],
            (gs.R_16F, gs.R_16F): [gs.COMPUTE_32F, gs.COMPUTE_16F],
            (gs.R_16BF, gs.R_32F): [gs.COMPUTE_32F, gs.COMPUTE_32F_FAST_16BF],
            (gs.R_16BF, gs.R_16BF): [gs.COMPUTE_32F],
            (gs.R_8I, gs.R_32I): [gs.COMPUTE_32I, gs.COMPUTE_32I_PEDANTIC],
            (gs.R_32F, gs.R_32F): [gs.COMPUTE_32F, gs.COMPUTE_32F_FAST_TF32]}


def draw(i):
    rng = np.random.default_rng(1000 + i)
    dt = [gs.R_16F, gs.R_16BF, gs.R_8I, gs.R_32F][i % 4]
    ct = OUTS[dt][rng.integers(len(OUTS[dt]))]
    comp = COMPUTES[(dt, ct)][rng.integers(len(COMPUTES[(dt, ct)]))]
    # half the cases log-uniform in [1, 700] (edges, tiny shapes), half uniform in [128, 700] (full tiles)
    if i % 2:
        dims = [int(np.exp(rng.uniform(0, np.log(700)))) for _ in range(3)]
    else:
        dims = [int(rng.integers(128, 701)) for _ in range(3)]
    m, n, k = dims
    if rng.random() < 0.06:
        k = 0
    batch = int(rng.choice([1, 1, 2, 3]))
    while m * n * max(k, 1) * batch > 1.2e8:
        m, n = max(1, m // 2), max(1, n // 2)
    return dict(dt=dt, ct=ct, comp=comp, op_a=int(rng.integers(3)), op_b=int(rng.integers(3)), m=m, n=n, k=k,
                batch=batch, pads=[int(rng.choice([0, 0, 1, 3, 8, 16])) for _ in range(3)],
                spads=[int(rng.choice([0, 0, 5, 64])) for _ in range(3)], ptr=batch > 1 and rng.random() < 0.35,
                algo=int(rng.choice([-1, -1, 0, 1, 2])), alpha=(float(rng.integers(-3, 4)) if dt == gs.R_8I
                                                                else float(rng.uniform(-2, 2))),
                beta=(float(rng.choice([0, 0, 1, -2])) if dt == gs.R_8I else float(rng.choice([0.0, 0.0, 0.5, -1.25]))),
                seed=int(rng.integers(1 << 30)))


def ext(rows, cols, ld):
    return (cols - 1) * ld + rows if rows and cols else 0


@pytest.mark.parametrize("i", range(N_CASES))
def test_random_case(handle, i):
    import torch

    c = draw(i)
    dt, ct, comp, m, n, k, batch = c["dt"], c["ct"], c["comp"], c["m"], c["n"], c["k"], c["batch"]
    op_a, op_b = c["op_a"], c["op_b"]
    rng = np.random.default_rng(c["seed"])
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    lda, ldb, ldc = max(1, ar) + c["pads"][0], max(1, br) + c["pads"][1], max(1, m) + c["pads"][2]
    sa = ext(ar, ac, lda) + c["spads"][0]
    sb = ext(br, bc, ldb) + c["spads"][1]
    sc = ext(m, n, ldc) + c["spads"][2]
    a = make_input(rng, max(1, sa * batch), dt)
    b = make_input(rng, max(1, sb * batch), dt)
    c0 = make_c(rng, max(1, sc * batch), ct)
    ref = c0.copy()
    if c["ptr"]:
        da, db, dc = to_dev(a), to_dev(b), to_dev(c0)
        es, ec = np.dtype(NP_OF[dt]).itemsize, np.dtype(NP_OF[ct]).itemsize
        arr = lambda t, stride, e: torch.tensor([t.data_ptr() + j * stride * e for j in range(batch)],  # noqa
                                                dtype=torch.int64, device="cuda")
        handle.gemm_batched_ex(op_a, op_b, m, n, k, c["alpha"], arr(da, sa, es), dt, lda, arr(db, sb, es), dt, ldb,
                               c["beta"], arr(dc, sc, ec), ct, ldc, batch, comp, algo=c["algo"])
        got = to_host(dc)
        a_l = [a[j * sa:j * sa + max(1, ext(ar, ac, lda))] for j in range(batch)]
        b_l = [b[j * sb:j * sb + max(1, ext(br, bc, ldb))] for j in range(batch)]
        c_l = [ref[j * sc:j * sc + max(1, ext(m, n, ldc))].copy() for j in range(batch)]
        assert orc.gemm_batched_ex(op_a, op_b, m, n, k, c["alpha"], a_l, dt, lda, b_l, dt, ldb, c["beta"], c_l, ct,
                                   ldc, compute_type=comp) == orc.OK
        for j in range(batch):
            ref[j * sc:j * sc + len(c_l[j])] = c_l[j]
    else:
        da, db, dc = to_dev(a), to_dev(b), to_dev(c0)
        handle.gemm_strided_batched_ex(op_a, op_b, m, n, k, c["alpha"], da, dt, lda, sa, db, dt, ldb, sb, c["beta"],
                                       dc, ct, ldc, sc, batch, comp, algo=c["algo"])
        got = to_host(dc)
        assert orc.gemm_ex(op_a, op_b, m, n, k, c["alpha"], a, dt, lda, b, dt, ldb, c["beta"], ref, ct, ldc,
                           compute_type=comp, batch=batch, sa=sa, sb=sb, sc=sc, threads=8) == orc.OK
    mask = np.zeros(c0.size, dtype=bool)
    if m and n:
        idx = (np.arange(batch)[:, None, None] * sc + np.arange(n)[None, :, None] * ldc +
               np.arange(m)[None, None, :]).ravel()
        mask[idx] = True
    tol_dt = gs.R_32F if dt == gs.R_8I else dt
    if ct == gs.R_16F or ct == gs.R_16BF:
        tol_dt = ct
    assert_parity(got, ref, ct, tol_dt, mask=mask, c_before=c0)
    assert handle.device_error() == 0, c


def draw_tf32(i):
    rng = np.random.default_rng(5000 + i)
    while True:
        m, n = int(rng.integers(128, 2049)), int(rng.integers(128, 2049))
        k = int(np.exp(rng.uniform(np.log(64), np.log(4000))))
        batch = int(rng.choice([1, 1, 2]))
        flops = 2.0 * m * n * k * batch
        if 1.0e9 <= flops <= 4.0e9:
            break
    return dict(m=m, n=n, k=k, batch=batch, op_a=int(rng.integers(3)), op_b=int(rng.integers(3)),
                pads=[int(rng.choice([0, 0, 1, 4])) for _ in range(3)], spads=[int(rng.choice([0, 8])) for _ in range(3)],
                alpha=float(rng.uniform(-2, 2)), beta=float(rng.choice([0.0, 0.5, -1.0])), seed=int(rng.integers(1 << 30)))


@pytest.mark.parametrize("i", range(24))
def test_random_fast_tf32_case(handle, i):
    """Seeded sweep of COMPUTE_32F_FAST_TF32 problems large enough for the tensor-core path (split operands, chunked
    kind::tf32 accumulation): ops, ragged shapes, padded leading dimensions and strides, batches, alpha / beta —
    each within the FP32 tolerance of the oracle, with C's padding untouched."""
    c = draw_tf32(i)
    m, n, k, batch, op_a, op_b = c["m"], c["n"], c["k"], c["batch"], c["op_a"], c["op_b"]
    rng = np.random.default_rng(c["seed"])
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    lda, ldb, ldc = ar + c["pads"][0], br + c["pads"][1], m + c["pads"][2]
    sa, sb, sc = ext(ar, ac, lda) + c["spads"][0], ext(br, bc, ldb) + c["spads"][1], ext(m, n, ldc) + c["spads"][2]
    a = make_input(rng, sa * batch, gs.R_32F)
    b = make_input(rng, sb * batch, gs.R_32F)
    c0 = make_c(rng, sc * batch, gs.R_32F)
    dc = to_dev(c0)
    handle.gemm_strided_batched_ex(op_a, op_b, m, n, k, c["alpha"], to_dev(a), gs.R_32F, lda, sa, to_dev(b), gs.R_32F,
                                   ldb, sb, c["beta"], dc, gs.R_32F, ldc, sc, batch, gs.COMPUTE_32F_FAST_TF32)
    assert handle.last_kernels() & gs.KERNEL_TC_TF32, c
    got = to_host(dc)
    ref = c0.copy()
    assert orc.gemm_ex(op_a, op_b, m, n, k, c["alpha"], a, gs.R_32F, lda, b, gs.R_32F, ldb, c["beta"], ref, gs.R_32F,
                       ldc, compute_type=gs.COMPUTE_32F_FAST_TF32, batch=batch, sa=sa, sb=sb, sc=sc,
                       threads=32) == orc.OK
    mask = np.zeros(c0.size, dtype=bool)
    idx = (np.arange(batch)[:, None, None] * sc + np.arange(n)[None, :, None] * ldc +
           np.arange(m)[None, None, :]).ravel()
    mask[idx] = True
    assert_parity(got, ref, gs.R_32F, gs.R_32F, mask=mask, c_before=c0)
    assert handle.device_error() == 0, c
