"""GPU parity of libgemm_sm100 against the CPU oracle, through the C ABI.

Each case builds seeded inputs on the host, runs the device entry point and
compares with the oracle's restatement of src/gemm.zig on the same bytes:
bit-exact for INT8 -> INT32, normwise relative error within 1e-5 (FP32),
2e-3 (FP16) and 1e-2 (BF16) otherwise. Sizes stay small enough for the
oracle to finish in seconds; full-size configurations are covered by
test_gpu_fullsize.py through sampled entries and exact checksums.
"""
import os

import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import COMPUTE, NP_OF, OUT_OF, TOL, assert_parity, make_c, make_input, to_dev, to_host

pytestmark = pytest.mark.gpu
THREADS = max(1, min(32, os.cpu_count() or 1))


def extent(rows, cols, ld):
    return 0 if rows == 0 or cols == 0 else (cols - 1) * ld + rows


def run_case(handle, dt, op_a, op_b, m, n, k, alpha=1.0, beta=0.0, ct=None, pad=(0, 0, 0), batch=1,
             stride_pad=(0, 0, 0), seed=0, expect_kernel=None, bcast_a=False, algo=gs.GEMM_DEFAULT, comp=None):
    """Runs one (strided-batched) gemmEx on the GPU and on the oracle; returns the kernel bits used."""
    rng = np.random.default_rng(seed)
    ct = OUT_OF[dt] if ct is None else ct
    comp = COMPUTE[dt] if comp is None else comp
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    lda, ldb, ldc = max(1, ar) + pad[0], max(1, br) + pad[1], max(1, m) + pad[2]
    sa = extent(ar, ac, lda) + stride_pad[0]
    sb = extent(br, bc, ldb) + stride_pad[1]
    sc = extent(m, n, ldc) + stride_pad[2]
    if bcast_a:
        sa = 0
    a = make_input(rng, max(1, sa * batch if sa else extent(ar, ac, lda)), dt)
    b = make_input(rng, max(1, sb * batch), dt)
    c = make_c(rng, max(1, sc * batch), ct)
    da, db, dc = to_dev(a), to_dev(b), to_dev(c)
    if batch == 1:
        handle.gemm_ex(op_a, op_b, m, n, k, alpha, da, dt, lda, db, dt, ldb, beta, dc, ct, ldc, comp, algo=algo)
    else:
        handle.gemm_strided_batched_ex(op_a, op_b, m, n, k, alpha, da, dt, lda, sa, db, dt, ldb, sb, beta, dc, ct,
                                       ldc, sc, batch, comp, algo=algo)
    kernels = handle.last_kernels()
    got = to_host(dc)
    ref = c.copy()
    if bcast_a:
        # the oracle has no broadcast stride: replicate A per batch
        a_rep = np.concatenate([a[:extent(ar, ac, lda)]] * batch)
        rc = orc.gemm_ex(op_a, op_b, m, n, k, alpha, a_rep, dt, lda, b, dt, ldb, beta, ref, ct, ldc,
                         compute_type=comp, batch=batch, sa=extent(ar, ac, lda), sb=sb, sc=sc, threads=THREADS)
    else:
        rc = orc.gemm_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, ref, ct, ldc, compute_type=comp,
                         batch=batch, sa=sa, sb=sb, sc=sc, threads=THREADS)
    assert rc == orc.OK
    mask = np.zeros(c.size, dtype=bool)
    if m and n:
        idx = (np.arange(batch)[:, None, None] * sc + np.arange(n)[None, :, None] * ldc +
               np.arange(m)[None, None, :]).ravel()
        mask[idx] = True
    assert_parity(got, ref, ct, dt if dt != gs.R_8I else gs.R_32F, mask=mask, c_before=c)
    if expect_kernel is not None:
        assert kernels & expect_kernel, (kernels, expect_kernel)
    assert handle.device_error() == 0
    return kernels


TC = {gs.R_16F: gs.KERNEL_TC_F16, gs.R_16BF: gs.KERNEL_TC_BF16, gs.R_8I: gs.KERNEL_TC_I8}
# algo hint: 0 = 1-SM 128x256 tile, 1 = 2-SM 256x256 pair tile, 2 = 2-SM 256x512 wide pair tile
# (results must not depend on it)
TILES = [0, 1, 2]


@pytest.mark.parametrize("algo", TILES)
@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_16BF, gs.R_8I])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_tc_exact_tiles(handle, dt, op_a, op_b, algo):
    run_case(handle, dt, op_a, op_b, 512, 512, 512, seed=1, expect_kernel=TC[dt], algo=algo)


@pytest.mark.parametrize("algo", TILES)
@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_16BF, gs.R_8I])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_tc_ragged_edges_alpha_beta(handle, dt, op_a, op_b, algo):
    # M, N, K not multiples of the 256 x 256 x (64|128) tile; alpha/beta applied.
    q = 16 if dt == gs.R_8I else 8
    m, n, k = 41 * q, 37 * q, 11 * q
    alpha, beta = (2.0, -1.0) if dt == gs.R_8I else (1.5, 0.5)
    run_case(handle, dt, op_a, op_b, m, n, k, alpha=alpha, beta=beta, seed=2, expect_kernel=TC[dt], algo=algo)


@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I])
def test_tc_small_m_and_single_tile(handle, dt):
    # M <= 128 picks the 1-SM tile automatically; M = 136 leaves the odd CTA 8 rows.
    q = 16 if dt == gs.R_8I else 8
    run_case(handle, dt, 0, 0, 64, 256, 128, seed=3, expect_kernel=TC[dt])
    run_case(handle, dt, 1, 0, 17 * q, 2 * q, 3 * q, seed=3, expect_kernel=TC[dt], algo=1)
    run_case(handle, dt, 0, 1, 128, 1024, 4 * q, seed=3, expect_kernel=TC[dt], algo=1)


@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I])
def test_tc_padded_leading_dimensions(handle, dt):
    q = 16 if dt == gs.R_8I else 8
    run_case(handle, dt, 0, 0, 160, 300, 192, pad=(q, 2 * q, 5), seed=3, expect_kernel=TC[dt])
    run_case(handle, dt, 1, 1, 160, 304, 192, pad=(q, q, 3), alpha=3.0 if dt == gs.R_8I else 0.25,
             beta=1.0 if dt == gs.R_8I else -2.0, seed=4, expect_kernel=TC[dt])


@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_16BF, gs.R_8I, gs.R_32F])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 1), (2, 0)])
def test_unaligned_shapes_use_cuda_core_kernel(handle, dt, op_a, op_b):
    # odd sizes leave leading dimensions off the 16-byte grid TMA needs
    kern = run_case(handle, dt, op_a, op_b, 37, 41, 29, alpha=2.0 if dt == gs.R_8I else 1.25,
                    beta=-1.0 if dt == gs.R_8I else 0.5, pad=(1, 3, 2), seed=5)
    if dt == gs.R_32F:
        assert kern & gs.KERNEL_FFMA
    else:
        assert kern & gs.KERNEL_SIMT


@pytest.mark.parametrize("algo", TILES)
@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_16BF, gs.R_8I])
def test_strided_batched(handle, dt, algo):
    q = 16 if dt == gs.R_8I else 8
    run_case(handle, dt, 0, 0, 256, 256, 192, batch=5, seed=6, expect_kernel=TC[dt], algo=algo)
    run_case(handle, dt, 1, 0, 96, 136, 64, batch=3, stride_pad=(q, 2 * q, 7), alpha=2.0 if dt == gs.R_8I else 0.5,
             beta=1.0 if dt == gs.R_8I else 0.25, seed=7, expect_kernel=TC[dt], algo=algo)
    run_case(handle, dt, 0, 1, 384, 128, 128, batch=4, bcast_a=True, seed=8, expect_kernel=TC[dt], algo=algo)


def test_strided_batched_config4_shape_small_batch(handle):
    # the configuration-4 GEMM shape (512 x 512 x 1024, alpha = 1/sqrt(K)) at batch 6
    run_case(handle, gs.R_16F, 0, 0, 512, 512, 1024, alpha=1.0 / 32.0, batch=6, seed=9, expect_kernel=gs.KERNEL_TC_F16)


@pytest.mark.parametrize("ct", [gs.R_16F, gs.R_16BF])
def test_low_precision_outputs(handle, ct):
    dt = gs.R_16F if ct == gs.R_16F else gs.R_16BF
    run_case(handle, dt, 0, 0, 136, 264, 128, ct=ct, alpha=1.5, beta=0.5, seed=10, expect_kernel=TC[dt])
    run_case(handle, dt, 1, 1, 64, 40, 24, ct=ct, pad=(1, 1, 1), seed=11, expect_kernel=gs.KERNEL_SIMT)


def test_hgemm_matches_oracle_hgemm(handle):
    rng = np.random.default_rng(12)
    m, n, k = 192, 264, 136
    a = orc.randn_lowp(rng, m * k, orc.R_16F)
    b = orc.randn_lowp(rng, k * n, orc.R_16F)
    c = orc.randn_lowp(rng, m * n, orc.R_16F)
    dc = to_dev(c)
    handle.hgemm(0, 1, m, n, k, 1.5, to_dev(a), m, to_dev(b), n, -0.5, dc, m)
    assert handle.last_kernels() & gs.KERNEL_TC_F16
    ref = c.copy()
    assert orc.hgemm(orc.COL_MAJOR, 0, 1, m, n, k, orc.f32_to_f16_bits(1.5), a, m, b, n, orc.f32_to_f16_bits(-0.5),
                     ref, m) == orc.OK
    assert_parity(to_host(dc), ref, gs.R_16F, gs.R_16F)


@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I, gs.R_32F])
def test_k_zero_applies_beta_only(handle, dt):
    ct = OUT_OF[dt]
    rng = np.random.default_rng(13)
    m, n = 70, 50
    c = make_c(rng, m * n, ct)
    dc = to_dev(c)
    dummy = to_dev(np.zeros(16, NP_OF[dt]))
    beta = 3.0 if dt == gs.R_8I else 0.5
    handle.gemm_ex(0, 0, m, n, 0, 2.0, dummy, dt, m, dummy, dt, 1, beta, dc, ct, m, COMPUTE[dt])
    assert handle.last_kernels() == gs.KERNEL_SCALE
    ref = c.copy()
    assert orc.gemm_ex(0, 0, m, n, 0, 2.0, np.zeros(1, NP_OF[dt]), dt, m, np.zeros(1, NP_OF[dt]), dt, 1, beta, ref,
                       ct, m, compute_type=COMPUTE[dt]) == orc.OK
    assert_parity(to_host(dc), ref, ct, gs.R_32F)


def test_empty_shapes_are_noops(handle):
    c = to_dev(np.full(8, 7.0, np.float32))
    dummy = to_dev(np.zeros(8, np.uint16))
    handle.gemm_ex(0, 0, 0, 4, 4, 1.0, dummy, gs.R_16F, 1, dummy, gs.R_16F, 4, 0.0, c, gs.R_32F, 1, gs.COMPUTE_32F)
    handle.gemm_strided_batched_ex(0, 0, 2, 4, 4, 1.0, dummy, gs.R_16F, 2, 8, dummy, gs.R_16F, 4, 16, 0.0, c,
                                   gs.R_32F, 2, 8, 0, gs.COMPUTE_32F)
    assert handle.last_kernels() == 0
    np.testing.assert_array_equal(to_host(c), np.full(8, 7.0, np.float32))


def test_error_statuses_on_device_handle(handle):
    dummy = to_dev(np.zeros(64, np.uint16))
    s = handle.gemm_ex(0, 0, 4, 4, 4, 1.0, dummy, gs.R_16F, 2, dummy, gs.R_16F, 4, 0.0, dummy, gs.R_32F, 4,
                       gs.COMPUTE_32F, check=False)
    assert s == gs.STATUS_INVALID_VALUE and "lda" in handle.last_error()
    s = handle.gemm_ex(0, 0, 4, 4, 4, 1.0, dummy, gs.R_16F, 4, dummy, gs.R_16BF, 4, 0.0, dummy, gs.R_32F, 4,
                       gs.COMPUTE_32F, check=False)
    assert s == gs.STATUS_NOT_SUPPORTED
    with pytest.raises(gs.GemmError):
        handle.gemm_ex(0, 0, -1, 4, 4, 1.0, dummy, gs.R_16F, 4, dummy, gs.R_16F, 4, 0.0, dummy, gs.R_32F, 4,
                       gs.COMPUTE_32F)


# ---- SGEMM (FFMA) -----------------------------------------------------------

def sgemm_case(handle, op_a, op_b, m, n, k, alpha, beta, pad=(0, 0, 0), seed=0):
    rng = np.random.default_rng(seed)
    ar, ac = (m, k) if op_a == 0 else (k, m)
    br, bc = (k, n) if op_b == 0 else (n, k)
    lda, ldb, ldc = ar + pad[0], br + pad[1], m + pad[2]
    a = rng.uniform(-1, 1, (ac - 1) * lda + ar).astype(np.float32)
    b = rng.uniform(-1, 1, (bc - 1) * ldb + br).astype(np.float32)
    c = rng.uniform(-1, 1, (n - 1) * ldc + m).astype(np.float32)
    dc = to_dev(c)
    handle.sgemm(op_a, op_b, m, n, k, alpha, to_dev(a), lda, to_dev(b), ldb, beta, dc, ldc)
    assert handle.last_kernels() == gs.KERNEL_FFMA
    ref = c.copy()
    assert orc.sgemm_strided_batched_mt(orc.COL_MAJOR, op_a, op_b, m, n, k, alpha, a, lda, 0, b, ldb, 0, beta, ref,
                                        ldc, 0, 1, THREADS) == orc.OK
    mask = np.zeros(c.size, bool)
    mask[(np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).ravel()] = True
    return assert_parity(to_host(dc), ref, gs.R_32F, gs.R_32F, mask=mask, c_before=c)


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("shape", [(1024, 4096, 512), (4096, 1024, 2048)])
def test_sgemm_config2(handle, op_a, op_b, shape):
    m, n, k = shape
    sgemm_case(handle, op_a, op_b, m, n, k, 1.5, 0.5, seed=20)


def test_sgemm_config1_and_edges(handle):
    sgemm_case(handle, 0, 0, 512, 512, 512, 1.0, 0.0, seed=21)
    sgemm_case(handle, 1, 0, 130, 70, 33, -0.75, 0.25, pad=(3, 1, 2), seed=22)
    sgemm_case(handle, 0, 1, 5, 4, 3, 1.25, -0.5, pad=(1, 2, 1), seed=23)
    sgemm_case(handle, 2, 2, 257, 129, 9, 1.0, 1.0, seed=24)


@pytest.mark.parametrize("op_b", [0, 1])
def test_sgemm_wider_than_one_grid(handle, op_b):
    """More than 65535 * 32 output columns: the FFMA launcher cuts C (and B) into column slices, each one grid."""
    sgemm_case(handle, 0, op_b, 8, 2_200_000, 4, 1.25, 0.5, seed=26 + op_b)


def test_sgemm_strided_batched(handle):
    rng = np.random.default_rng(25)
    m, n, k, batch = 96, 80, 40, 3
    a = rng.uniform(-1, 1, m * k * batch).astype(np.float32)
    b = rng.uniform(-1, 1, k * n * batch).astype(np.float32)
    c = rng.uniform(-1, 1, m * n * batch).astype(np.float32)
    dc = to_dev(c)
    handle.sgemm_strided_batched(0, 1, m, n, k, 1.5, to_dev(a), m, m * k, to_dev(b), n, k * n, 0.5, dc, m, m * n,
                                 batch)
    ref = c.copy()
    assert orc.sgemm_strided_batched_mt(orc.COL_MAJOR, 0, 1, m, n, k, 1.5, a, m, m * k, b, n, k * n, 0.5, ref, m,
                                        m * n, batch, THREADS) == orc.OK
    assert_parity(to_host(dc), ref, gs.R_32F, gs.R_32F)



# ---- split-K: long-K single GEMMs whose tiles fill under half the SMs ----------

@pytest.mark.parametrize("dt,ct,op_a,op_b,m,n,k,alpha,beta,pad", [
    (gs.R_16F, gs.R_32F, 0, 0, 512, 512, 16384, 1.0, 0.0, (0, 0, 0)),        # 16 slices of 1024
    (gs.R_16BF, gs.R_16BF, 1, 0, 512, 512, 16384, 0.75, -0.5, (0, 0, 0)),   # bf16 output rounded once, after the sum
    (gs.R_8I, gs.R_32I, 0, 1, 384, 640, 8192, 2.0, -1.0, (0, 0, 0)),        # INT8: exact s32 sums, clamped epilogue
    (gs.R_16F, gs.R_16F, 1, 1, 264, 200, 8192, 1.25, 0.5, (0, 0, 0)),       # ragged M and N, f16 output
    (gs.R_16F, gs.R_32F, 0, 0, 1024, 1024, 4096, 1.5, 0.25, (0, 0, 0)),     # 4 slices
    (gs.R_16F, gs.R_32F, 0, 1, 512, 512, 16384, 1.0, 0.5, (8, 16, 3)),      # padded lda / ldb / ldc, beta != 0
    (gs.R_8I, gs.R_32I, 1, 0, 512, 256, 16384, 3.0, 2.0, (16, 32, 5)),      # padded, INT8, ldc not a multiple of 4
])
def test_splitk_matches_oracle(handle, dt, ct, op_a, op_b, m, n, k, alpha, beta, pad):
    """Long-K GEMMs with few output tiles split K into slices that run as a strided batch of the tensor-core
    kernel into a workspace; a second kernel adds the slices in order and applies alpha / beta with the
    reference's rounding. Bit-exact for INT8, within the type's tolerance otherwise, bytes outside C kept."""
    comp = gs.COMPUTE_32I if dt == gs.R_8I else gs.COMPUTE_32F
    kern = run_case(handle, dt, op_a, op_b, m, n, k, alpha=alpha, beta=beta, ct=ct, pad=pad, seed=m + n + k,
                    comp=comp, expect_kernel=TC[dt])
    assert kern & gs.KERNEL_REDUCE, kern


def test_splitk_not_taken_when_k_is_ragged_or_algo_is_forced(handle):
    """K that is not a whole number of stages, or an explicit tile hint, keeps the single launch."""
    kern = run_case(handle, gs.R_16F, 0, 0, 512, 512, 16384 + 8, seed=3, expect_kernel=gs.KERNEL_TC_F16)
    assert not kern & gs.KERNEL_REDUCE
    kern = run_case(handle, gs.R_16F, 0, 0, 512, 512, 16384, seed=4, algo=0, expect_kernel=gs.KERNEL_TC_F16)
    assert not kern & gs.KERNEL_REDUCE


# ---- pointer-array batches --------------------------------------------------

@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_16BF, gs.R_8I, gs.R_32F])
@pytest.mark.parametrize("misalign", [False, True])
@pytest.mark.parametrize("algo", TILES)
def test_pointer_array_batched(handle, dt, misalign, algo):
    import torch

    rng = np.random.default_rng(30 + dt)
    m, n, k, batch = 160, 264, 192, 5
    ct = OUT_OF[dt]
    es = np.dtype(NP_OF[dt]).itemsize
    shift = 1 if misalign else 0  # one element: breaks 16-byte alignment of every A pointer
    a_list = [make_input(rng, m * k + 8, dt) for _ in range(batch)]
    b_list = [make_input(rng, k * n, dt) for _ in range(batch)]
    c_list = [make_c(rng, m * n, ct) for _ in range(batch)]
    da = [to_dev(x) for x in a_list]
    db = [to_dev(x) for x in b_list]
    dc = [to_dev(x) for x in c_list]
    aptr = torch.tensor([t.data_ptr() + shift * es for t in da], dtype=torch.int64, device="cuda")
    bptr = torch.tensor([t.data_ptr() for t in db], dtype=torch.int64, device="cuda")
    cptr = torch.tensor([t.data_ptr() for t in dc], dtype=torch.int64, device="cuda")
    alpha, beta = (2.0, -1.0) if dt == gs.R_8I else (0.75, 0.5)
    handle.gemm_batched_ex(0, 0, m, n, k, alpha, aptr, dt, m, bptr, dt, k, beta, cptr, ct, m, batch, COMPUTE[dt],
                           algo=algo)
    kern = handle.last_kernels()
    refs = [x.copy() for x in c_list]
    a_view = [x[shift:shift + m * k].copy() for x in a_list]
    assert orc.gemm_batched_ex(0, 0, m, n, k, alpha, a_view, dt, m, b_list, dt, k, beta, refs, ct, m,
                               compute_type=COMPUTE[dt]) == orc.OK
    for i in range(batch):
        assert_parity(to_host(dc[i]), refs[i], ct, dt if dt != gs.R_8I else gs.R_32F)
    if dt == gs.R_32F:
        assert kern & gs.KERNEL_FFMA
    else:
        # up to PTR_MAPS_IN_KERNEL_MAX_BATCH entries the GEMM kernel builds its own maps: no builder launch
        assert kern & TC[dt] and not kern & gs.KERNEL_TMAP
    assert handle.device_error() == 0


@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I])
@pytest.mark.parametrize("batch", [gs.PTR_MAPS_IN_KERNEL_MAX_BATCH, gs.PTR_MAPS_IN_KERNEL_MAX_BATCH + 6])
@pytest.mark.parametrize("beta,misalign", [(0.5, None), (0.0, None), (0.0, "c"), (0.5, "a")])
@pytest.mark.parametrize("algo", TILES)
def test_pointer_array_map_paths(handle, dt, batch, beta, misalign, algo):
    """Both ways of building the per-entry tensor maps of a pointer-array call, against the oracle: at the
    in-kernel limit (one launch; each CTA writes its own maps) and past it (the map builder, then the GEMM: two
    launches), with TMA-stored C (beta 0), a misaligned C entry (direct stores), a misaligned A entry (CUDA-core
    fallback for the whole batch) and directly stored C (beta != 0). Ragged M and N."""
    import torch

    rng = np.random.default_rng(70 + dt + batch + algo + (misalign == "c") + 2 * (misalign == "a") + int(4 * beta))
    m, n, k = 144, 72, 64  # leading dimensions TMA can address for every type (16-byte multiples)
    ct = OUT_OF[dt]
    es_a, es_c = np.dtype(NP_OF[dt]).itemsize, np.dtype(NP_OF[ct]).itemsize
    a_list = [make_input(rng, m * k + 8, dt) for _ in range(batch)]
    b_list = [make_input(rng, k * n, dt) for _ in range(batch)]
    c_list = [make_c(rng, m * n + 8, ct) for _ in range(batch)]
    da, db, dc = [to_dev(x) for x in a_list], [to_dev(x) for x in b_list], [to_dev(x) for x in c_list]
    bad = batch - 3  # the entry whose A or C pointer is off by one element
    sa = [1 if misalign == "a" and j == bad else 0 for j in range(batch)]
    sc = [1 if misalign == "c" and j == bad else 0 for j in range(batch)]
    aptr = torch.tensor([t.data_ptr() + sa[j] * es_a for j, t in enumerate(da)], dtype=torch.int64, device="cuda")
    bptr = torch.tensor([t.data_ptr() for t in db], dtype=torch.int64, device="cuda")
    cptr = torch.tensor([t.data_ptr() + sc[j] * es_c for j, t in enumerate(dc)], dtype=torch.int64, device="cuda")
    alpha = 2.0 if dt == gs.R_8I else 0.75
    if dt == gs.R_8I and beta != 0.0:
        beta = -1.0  # COMPUTE_32I scalars are int32 (gemmEx's alpha/beta pointers)
    n0 = handle.launch_count()
    handle.gemm_batched_ex(0, 0, m, n, k, alpha, aptr, dt, m, bptr, dt, k, beta, cptr, ct, m, batch, COMPUTE[dt],
                           algo=algo)
    launched, kern = handle.launch_count() - n0, handle.last_kernels()
    refs = [x.copy() for x in c_list]
    views = [r[sc[j]:sc[j] + m * n] for j, r in enumerate(refs)]
    a_view = [x[sa[j]:sa[j] + m * k].copy() for j, x in enumerate(a_list)]
    assert orc.gemm_batched_ex(0, 0, m, n, k, alpha, a_view, dt, m, b_list, dt, k, beta, views, ct, m,
                               compute_type=COMPUTE[dt]) == orc.OK
    for j in range(batch):
        assert_parity(to_host(dc[j]), refs[j], ct, dt if dt != gs.R_8I else gs.R_32F)
    in_kernel = batch <= gs.PTR_MAPS_IN_KERNEL_MAX_BATCH
    assert kern & TC[dt]
    assert bool(kern & gs.KERNEL_TMAP) == (not in_kernel)
    assert launched == (1 if in_kernel else 2)
    assert handle.device_error() == 0


@pytest.mark.parametrize("dt,ct", [(gs.R_16F, gs.R_32F), (gs.R_16BF, gs.R_16BF), (gs.R_8I, gs.R_32I),
                                   (gs.R_16F, gs.R_16F)])
@pytest.mark.parametrize("c_shift_entry", [-1, 2])
@pytest.mark.parametrize("algo", TILES)
def test_pointer_array_tma_store_c(handle, dt, ct, c_shift_entry, algo):
    """beta == 0 pointer-array batches write C with TMA stores through per-entry C maps built on the device; a C
    entry that is not 16-byte aligned switches the whole call to direct stores. Ragged M/N, a padded ldc and bytes
    between columns (and past each entry) that must stay untouched."""
    import torch

    rng = np.random.default_rng(50 + dt + ct + algo)
    m, n, k, batch, pad = 300, 136, 96, 4, 8
    ldc = m + pad
    es_c = np.dtype(NP_OF[ct]).itemsize
    a_list = [make_input(rng, m * k, dt) for _ in range(batch)]
    b_list = [make_input(rng, k * n, dt) for _ in range(batch)]
    c_list = [make_c(rng, ldc * n + 16, ct) for _ in range(batch)]
    da = [to_dev(x) for x in a_list]
    db = [to_dev(x) for x in b_list]
    dc = [to_dev(x) for x in c_list]
    shift = [1 if j == c_shift_entry else 0 for j in range(batch)]  # one element: 2 or 4 bytes
    aptr = torch.tensor([t.data_ptr() for t in da], dtype=torch.int64, device="cuda")
    bptr = torch.tensor([t.data_ptr() for t in db], dtype=torch.int64, device="cuda")
    cptr = torch.tensor([t.data_ptr() + shift[j] * es_c for j, t in enumerate(dc)], dtype=torch.int64, device="cuda")
    comp = gs.COMPUTE_32I if dt == gs.R_8I else gs.COMPUTE_32F
    alpha = 3.0 if dt == gs.R_8I else 1.25
    handle.gemm_batched_ex(0, 0, m, n, k, alpha, aptr, dt, m, bptr, dt, k, 0.0, cptr, ct, ldc, batch, comp,
                           algo=algo)
    refs = [x.copy() for x in c_list]
    views = [r[shift[j]:] for j, r in enumerate(refs)]
    assert orc.gemm_batched_ex(0, 0, m, n, k, alpha, a_list, dt, m, b_list, dt, k, 0.0, views, ct, ldc,
                               compute_type=comp) == orc.OK
    for j in range(batch):
        got = to_host(dc[j])
        mask = np.zeros(got.size, bool)
        mask[shift[j] + (np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).ravel()] = True
        tol_dt = gs.R_32F if dt == gs.R_8I else (ct if ct in (gs.R_16F, gs.R_16BF) else dt)
        assert_parity(got, refs[j], ct, tol_dt, mask=mask, c_before=c_list[j])
    assert handle.device_error() == 0


# ---- host-buffer mirror of gemm.gemmEx --------------------------------------

@pytest.mark.parametrize("layout", [orc.COL_MAJOR, orc.ROW_MAJOR])
@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I])
def test_host_mirror_matches_oracle_gemm_ex(handle, layout, dt):
    rng = np.random.default_rng(40)
    m, n, k, batch = 72, 48, 40, 2
    ct = OUT_OF[dt]
    op_a, op_b = 1, 0
    # row-major lda is the stored column count
    ar, ac = (k, m)
    br, bc = (k, n)
    lda = (ac if layout == orc.ROW_MAJOR else ar) + 8
    ldb = (bc if layout == orc.ROW_MAJOR else br) + 16
    ldc = (n if layout == orc.ROW_MAJOR else m)
    ext = lambda r, c_, ld: (r - 1) * ld + c_ if layout == orc.ROW_MAJOR else (c_ - 1) * ld + r  # noqa: E731
    sa, sb, sc = ext(ar, ac, lda), ext(br, bc, ldb), ext(m, n, ldc)
    a = make_input(rng, sa * batch, dt)
    b = make_input(rng, sb * batch, dt)
    c = make_c(rng, sc * batch, ct)
    alpha, beta = (2.0, 1.0) if dt == gs.R_8I else (1.25, -0.5)
    got = c.copy()
    handle.host_gemm_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, got, ct, ldc, COMPUTE[dt],
                        layout=layout, batch=batch)
    ref = c.copy()
    assert orc.gemm_ex(op_a, op_b, m, n, k, alpha, a, dt, lda, b, dt, ldb, beta, ref, ct, ldc,
                       compute_type=COMPUTE[dt], layout=layout, batch=batch) == orc.OK
    assert_parity(got, ref, ct, dt if dt != gs.R_8I else gs.R_32F)


def test_host_mirror_validation(handle):
    a = np.zeros(6, np.uint16)
    c = np.zeros(4, np.float32)
    s = handle.host_gemm_ex(0, 0, 2, 2, 3, 1.0, a, gs.R_16F, 2, a, gs.R_16F, 3, 0.0, c, gs.R_32F, 2,
                            gs.COMPUTE_32F, batch=0, check=False)
    assert s == gs.STATUS_INVALID_VALUE and "InvalidBatchCount" in handle.last_error()
    s = handle.host_gemm_ex(0, 0, 2, 2, 3, 1.0, a, gs.R_16F, 2, a, gs.R_16F, 3, 0.0, c, gs.R_32F, 2,
                            gs.COMPUTE_32F, batch=2, check=False)
    assert s == gs.STATUS_INVALID_VALUE and "BufferTooSmall" in handle.last_error()


def test_stream_is_honoured(handle):
    import torch

    s = torch.cuda.Stream()
    handle.set_stream(s)
    try:
        with torch.cuda.stream(s):
            run_case(handle, gs.R_16F, 0, 0, 128, 256, 128, seed=50, expect_kernel=gs.KERNEL_TC_F16)
    finally:
        handle.set_stream(None)


# ---- TMA-store epilogue (beta == 0, C 16-byte addressable) ------------------

@pytest.mark.parametrize("algo", TILES)
@pytest.mark.parametrize("dt,ct", [(gs.R_16F, gs.R_32F), (gs.R_16F, gs.R_16F), (gs.R_16BF, gs.R_16BF),
                                   (gs.R_16BF, gs.R_32F), (gs.R_8I, gs.R_32I)])
def test_tma_store_epilogue_ragged(handle, dt, ct, algo):
    # beta = 0 with a TMA-addressable C routes the epilogue through TMA tensor
    # stores; ragged M / N exercise the clipping of partial 32 x 32 boxes.
    q = 16 if dt == gs.R_8I else 8
    alpha = 3.0 if dt == gs.R_8I else 0.75
    run_case(handle, dt, 0, 0, 37 * q, 45 * q, 9 * q, alpha=alpha, ct=ct, seed=60, expect_kernel=TC[dt], algo=algo)
    run_case(handle, dt, 1, 1, 19 * q, 13 * q, 5 * q, alpha=1.0, ct=ct, batch=3, stride_pad=(q, q, 8), seed=61,
             expect_kernel=TC[dt], algo=algo)


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 1), (0, 1)])
def test_fp32_fast_tf32_runs_exact_ffma(handle, op_a, op_b):
    """COMPUTE_32F_FAST_TF32 permits (does not require) TF32 products: this backend computes it exactly on the
    FFMA kernel, to the FP32 tolerance."""
    run_case(handle, gs.R_32F, op_a, op_b, 192, 160, 96, alpha=1.5, beta=0.5, seed=70, expect_kernel=gs.KERNEL_FFMA,
             comp=gs.COMPUTE_32F_FAST_TF32)


@pytest.mark.parametrize("op_a,op_b,m,n,k,batch,pad,bcast_a,kernel", [
    (0, 0, 2048, 1024, 256, 1, (0, 0, 0), False, gs.KERNEL_TC_TF32),
    (1, 0, 1536, 1024, 383, 1, (3, 1, 2), False, gs.KERNEL_TC_TF32),   # K not a multiple of 4, unaligned lds
    (0, 1, 1024, 2048, 300, 1, (0, 0, 0), False, gs.KERNEL_TC_TF32),
    (1, 1, 1024, 1024, 200, 3, (0, 0, 0), False, gs.KERNEL_TC_TF32),   # strided batch
    (0, 0, 1024, 2048, 256, 2, (0, 0, 0), True, gs.KERNEL_TC_TF32),    # broadcast A (stride 0)
    (2, 2, 1100, 1300, 350, 1, (1, 0, 5), False, gs.KERNEL_TC_TF32),   # op C, ragged tiles
    (0, 0, 1024, 512, 2048, 1, (0, 0, 0), False, gs.KERNEL_TC_TF32),   # 6 accumulator fills
    (1, 0, 768, 640, 1601, 2, (0, 2, 3), False, gs.KERNEL_TC_TF32),    # 5 fills, the last one partial; batched
    (0, 1, 128, 4096, 1200, 1, (0, 0, 0), False, gs.KERNEL_TC_TF32),   # M = 128: the 1-SM tile path
    (0, 0, 100, 512, 4096, 1, (0, 0, 0), False, gs.KERNEL_FFMA),       # output thinner than a 128-row tile
])
def test_fast_tf32_tensor_cores(handle, op_a, op_b, m, n, k, batch, pad, bcast_a, kernel):
    """COMPUTE_32F_FAST_TF32 on large problems runs tcgen05 kind::tf32 over the split operands (three tf32 products
    per f32 product; K accumulated in fills of 36 stages that the epilogue adds in TMEM with exact f32 adds) and must
    still meet the FP32 normwise tolerance against the oracle."""
    run_case(handle, gs.R_32F, op_a, op_b, m, n, k, alpha=1.5, beta=-0.5, pad=pad, batch=batch, bcast_a=bcast_a,
             seed=m + n + k + batch, comp=gs.COMPUTE_32F_FAST_TF32, expect_kernel=kernel)


@pytest.mark.parametrize("m,n,k", [(32, 32, 40), (96, 64, 33), (200, 136, 260), (1000, 1000, 64),
                                   (2040, 1288, 72)])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_sgemm_tile_sizes(handle, m, n, k, op_a, op_b):
    """The FFMA kernel's three CTA tiles (32x32, 64x64, 128x128, chosen by grid size) on ragged shapes."""
    run_case(handle, gs.R_32F, op_a, op_b, m, n, k, alpha=1.5, beta=0.5, seed=m + n + k, expect_kernel=gs.KERNEL_FFMA)


@pytest.mark.parametrize("m,n,k,batch,pad", [
    (512, 512, 512, 1, (0, 0, 0)),      # 64 tiles: K split over clusters of 4
    (64, 64, 4096, 1, (0, 0, 0)),       # one tile: clusters of 8
    (100, 300, 1000, 1, (0, 0, 0)),     # ragged M, N and K (62.5 K steps over 8 CTAs)
    (64, 64, 528, 1, (0, 0, 0)),        # 33 K steps over 8 CTAs: the last CTA has none
    (64, 64, 70, 1, (0, 0, 0)),         # 5 K steps: clusters of 2
    (200, 200, 512, 2, (0, 0, 0)),      # batched, clusters of 8
    (96, 72, 260, 1, (1, 3, 2)),        # leading dimensions not multiples of 4: scalar loads and stores
])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 1), (1, 0)])
def test_sgemm_cluster_split_k(handle, m, n, k, batch, pad, op_a, op_b):
    """Small FP32 problems split K across a thread-block cluster and reduce the partial tiles through
    distributed shared memory; the result must match the oracle to the FP32 tolerance, with alpha and beta
    applied once, and bytes outside C unchanged."""
    run_case(handle, gs.R_32F, op_a, op_b, m, n, k, alpha=1.5, beta=-0.5, pad=pad, batch=batch, seed=m * n + k,
             expect_kernel=gs.KERNEL_FFMA)


@pytest.mark.parametrize("m,n,k,batch,pad", [
    (2100, 1300, 1100, 1, (0, 0, 0)),   # 187 tiles of 128 x 128 on 296 slots: ragged M, N and K, 69 K steps
    (1500, 1100, 1030, 2, (0, 0, 0)),   # batched: 216 tiles, 65 K steps
    (2048, 1536, 1040, 1, (1, 3, 2)),   # leading dimensions not multiples of 4: scalar loads and stores
    (4096, 1024, 2048, 1, (0, 0, 0)),   # C2's shape: 256 tiles, each split over two CTAs
])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 1), (1, 0)])
def test_sgemm_stream_k(handle, m, n, k, batch, pad, op_a, op_b):
    """FP32 problems whose 128 x 128 tiles fill less than two waves of the resident CTA slots, leaving some
    idle, run stream-K (op T/N stays data-parallel): every CTA takes an equal share of the (tile, K step)
    iterations and the last contributor to a split tile sums the partial tiles in K order. The result must
    match the oracle to the FP32 tolerance, twice in a row on the same handle (the per-tile counters reset
    themselves), with alpha and beta applied once and bytes outside C unchanged."""
    for rep in range(2):
        run_case(handle, gs.R_32F, op_a, op_b, m, n, k, alpha=1.5, beta=-0.5, pad=pad, batch=batch,
                 seed=m + n + k + rep, expect_kernel=gs.KERNEL_FFMA)


