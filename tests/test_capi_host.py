"""CPU tests of libgemm_sm100's host logic: symbols, status codes, argument
validation and kernel choice (gs_plan_gemm_strided_batched_ex), shard
planning. No compute call is made here; see test_gpu_*.py for those."""
import ctypes
import subprocess

import pytest

import gemm_sm100 as gs
from conftest import gpu_available

ALIGNED = 1 << 20          # fake 16-byte aligned device addresses (never dereferenced)
ALIGNED_B = 2 << 20
ALIGNED_C = 3 << 20


def test_library_exports_every_declared_symbol():
    declared = gs.declared_symbols()
    assert len(declared) >= 18
    out = subprocess.run(["nm", "-D", "--defined-only", gs.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(gs.lib(), s)


def test_status_names():
    assert gs.status_name(0) == "GS_STATUS_SUCCESS"
    assert gs.status_name(7) == "GS_STATUS_INVALID_VALUE"
    assert gs.status_name(15) == "GS_STATUS_NOT_SUPPORTED"
    assert gs.status_name(12345) == "GS_STATUS_UNKNOWN"


def test_null_handle_is_not_initialized():
    L = gs.lib()
    one = ctypes.c_float(1.0)
    assert L.gs_sgemm(None, 0, 0, 4, 4, 4, ctypes.byref(one), ALIGNED, 4, ALIGNED, 4, ctypes.byref(one), ALIGNED,
                      4) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_gemm_ex(None, 0, 0, 4, 4, 4, ctypes.byref(one), ALIGNED, gs.R_16F, 4, ALIGNED, gs.R_16F, 4,
                        ctypes.byref(one), ALIGNED, gs.R_32F, 4, gs.COMPUTE_32F, -1) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_set_stream(None, None) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_host_gemm_ex(None, None) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_host_gemm_batched_ex(None, None) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_destroy(None) == gs.STATUS_NOT_INITIALIZED


@pytest.mark.skipif(gpu_available(), reason="checks behaviour without a GPU")
def test_create_without_gpu_fails_cleanly():
    h = ctypes.c_void_p()
    s = gs.lib().gs_create(ctypes.byref(h))
    assert s in (gs.STATUS_NOT_INITIALIZED, gs.STATUS_ARCH_MISMATCH)
    assert not h.value
    with pytest.raises(gs.GemmError):
        gs.Handle()


def plan(transa=0, transb=0, m=256, n=256, k=256, A=ALIGNED, at=gs.R_16F, lda=None, sa=0, B=ALIGNED_B, bt=None,
         ldb=None, sb=0, C=ALIGNED_C, ct=gs.R_32F, ldc=None, sc=0, batch=1, comp=gs.COMPUTE_32F):
    bt = at if bt is None else bt
    lda = (m if transa == 0 else k) if lda is None else lda
    ldb = (k if transb == 0 else n) if ldb is None else ldb
    ldc = m if ldc is None else ldc
    return gs.plan_gemm(transa, transb, m, n, k, A, at, lda, sa, B, bt, ldb, sb, C, ct, ldc, sc, batch, comp)


def test_plan_kernel_choice():
    assert plan() == (0, gs.KERNEL_TC_F16)
    assert plan(at=gs.R_16BF) == (0, gs.KERNEL_TC_BF16)
    assert plan(at=gs.R_8I, ct=gs.R_32I, comp=gs.COMPUTE_32I) == (0, gs.KERNEL_TC_I8)
    assert plan(at=gs.R_32F) == (0, gs.KERNEL_FFMA)
    assert plan(at=gs.R_16F, ct=gs.R_16F, comp=gs.COMPUTE_16F) == (0, gs.KERNEL_TC_F16)
    for ta in (0, 1, 2):
        for tb in (0, 1, 2):
            assert plan(transa=ta, transb=tb) == (0, gs.KERNEL_TC_F16)
    # k == 0 applies beta only; empty outputs launch nothing
    assert plan(k=0, lda=256, ldb=1) == (0, gs.KERNEL_SCALE)
    assert plan(m=0, ldc=1, lda=1) == (0, 0)
    assert plan(n=0) == (0, 0)
    assert plan(batch=0) == (0, 0)


def test_plan_fast_tf32_uses_tensor_cores_when_large():
    big = dict(at=gs.R_32F, ct=gs.R_32F, comp=gs.COMPUTE_32F_FAST_TF32, m=2048, n=2048, k=256, lda=2048, ldb=256,
               ldc=2048)
    assert plan(**big) == (0, gs.KERNEL_TC_TF32)
    # exact FP32 compute never takes the tf32 path
    assert plan(**{**big, "comp": gs.COMPUTE_32F}) == (0, gs.KERNEL_FFMA)
    # small problems and outputs thinner than a 128-row tile stay on FFMA; any K is fine (chunked accumulation)
    assert plan(at=gs.R_32F, ct=gs.R_32F, comp=gs.COMPUTE_32F_FAST_TF32) == (0, gs.KERNEL_FFMA)
    assert plan(**{**big, "m": 96, "lda": 96, "ldc": 96, "n": 65536}) == (0, gs.KERNEL_FFMA)
    assert plan(**{**big, "k": 8192, "ldb": 8192}) == (0, gs.KERNEL_TC_TF32)
    # unaligned leading dimensions are fine: the split kernel reads any layout
    assert plan(**{**big, "lda": 2051}) == (0, gs.KERNEL_TC_TF32)


def test_plan_falls_back_when_tma_cannot_address():
    # leading dimension not a multiple of 16 bytes
    assert plan(m=100, n=64, k=64, lda=100 + 3) == (0, gs.KERNEL_SIMT)
    # unaligned base pointer
    assert plan(A=ALIGNED + 2) == (0, gs.KERNEL_SIMT)
    # batch stride not a multiple of 16 bytes
    assert plan(batch=2, sa=256 * 256 + 4, sb=256 * 256) == (0, gs.KERNEL_SIMT)
    # stride 0 (broadcast) is fine
    assert plan(batch=4, sa=0, sb=256 * 256, sc=256 * 256) == (0, gs.KERNEL_TC_F16)
    # int8 rows must be 16-byte multiples
    assert plan(at=gs.R_8I, ct=gs.R_32I, comp=gs.COMPUTE_32I, m=200, lda=200) == (0, gs.KERNEL_SIMT)
    assert plan(at=gs.R_8I, ct=gs.R_32I, comp=gs.COMPUTE_32I, m=208, lda=208) == (0, gs.KERNEL_TC_I8)


def test_plan_validation_statuses():
    assert plan(transa=3)[0] == gs.STATUS_INVALID_VALUE
    assert plan(m=-1)[0] == gs.STATUS_INVALID_VALUE
    assert plan(batch=-1)[0] == gs.STATUS_INVALID_VALUE
    assert plan(lda=255)[0] == gs.STATUS_INVALID_VALUE
    assert plan(transa=1, lda=255)[0] == gs.STATUS_INVALID_VALUE
    assert plan(ldb=255)[0] == gs.STATUS_INVALID_VALUE
    assert plan(ldc=255)[0] == gs.STATUS_INVALID_VALUE
    assert plan(C=0)[0] == gs.STATUS_INVALID_VALUE
    assert plan(A=0)[0] == gs.STATUS_INVALID_VALUE
    # unsupported type / compute combinations
    assert plan(at=gs.R_16F, bt=gs.R_16BF)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(at=gs.R_8I, ct=gs.R_32F, comp=gs.COMPUTE_32F)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(at=gs.R_64F, ct=gs.R_64F, comp=gs.COMPUTE_64F)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(at=gs.R_16F, ct=gs.R_32F, comp=gs.COMPUTE_32I)[0] == gs.STATUS_NOT_SUPPORTED
    # int8 accumulator bound
    big = 131072
    assert plan(at=gs.R_8I, ct=gs.R_32I, comp=gs.COMPUTE_32I, k=big)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(at=gs.R_8I, ct=gs.R_32I, comp=gs.COMPUTE_32I, k=big - 1 - 15)[0] == 0
    # 32-bit tile coordinates: m, n, k above 2^31 - 1025 are refused, empty problems stay no-ops
    top = 2**31 - 1
    lim = top - 1024
    assert plan(m=lim + 1, lda=lim + 1, ldc=lim + 1)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(m=lim, lda=lim, ldc=lim)[0] == 0
    assert plan(n=top)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(k=lim + 1, ldb=lim + 1)[0] == gs.STATUS_NOT_SUPPORTED
    assert plan(k=lim, ldb=lim)[0] == 0
    assert plan(m=top, n=0, lda=top, ldc=top) == (0, 0)
    assert plan(m=top, lda=top - 1, ldc=top)[0] == gs.STATUS_INVALID_VALUE  # ld errors come first


@pytest.mark.parametrize("units,parts,align", [(256, 1, 1), (256, 8, 1), (64, 8, 1), (8192, 3, 256), (10, 4, 1),
                                               (3, 8, 1), (0, 2, 1), (8192, 8, 256)])
def test_plan_shards(units, parts, align):
    cuts = gs.plan_shards(units, parts, align)
    assert len(cuts) == parts + 1 and cuts[0] == 0 and cuts[-1] == units
    assert all(cuts[i] <= cuts[i + 1] for i in range(parts))
    assert all(c % align == 0 for c in cuts[:-1])
    if align == 1:
        assert cuts == [units * g // parts for g in range(parts)] + [units]


def test_plan_shards_rejects_bad_args():
    with pytest.raises(gs.GemmError):
        gs.plan_shards(-1, 2)
    with pytest.raises(gs.GemmError):
        gs.plan_shards(8, 0)


def test_multi_handle_argument_checks():
    """gs_multi_* reject bad arguments before touching any device."""
    L = gs.lib()
    h = ctypes.c_void_p()
    two = (ctypes.c_int * 2)(0, 0)
    assert L.gs_multi_create(None, 1, two) == gs.STATUS_INVALID_VALUE
    assert L.gs_multi_create(ctypes.byref(h), 0, two) == gs.STATUS_INVALID_VALUE
    assert L.gs_multi_create(ctypes.byref(h), 1, None) == gs.STATUS_INVALID_VALUE
    assert L.gs_multi_create(ctypes.byref(h), 2, two) == gs.STATUS_INVALID_VALUE       # duplicate device
    neg = (ctypes.c_int * 1)(-1)
    assert L.gs_multi_create(ctypes.byref(h), 1, neg) == gs.STATUS_INVALID_VALUE
    assert L.gs_multi_create(ctypes.byref(h), 65, (ctypes.c_int * 65)(*range(65))) == gs.STATUS_INVALID_VALUE
    assert not h.value
    assert L.gs_multi_destroy(None) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_multi_last_times(None, None, None) == gs.STATUS_NOT_INITIALIZED
    one = ctypes.c_float(1.0)
    ptrs = (ctypes.c_void_p * 1)(ALIGNED)
    assert L.gs_gemm_strided_batched_ex_multi(None, 0, 0, 4, 4, 4, ctypes.byref(one), ptrs, gs.R_16F, 4, 16, ptrs,
                                              gs.R_16F, 4, 16, ctypes.byref(one), ptrs, gs.R_32F, 4, 16, 2,
                                              gs.COMPUTE_32F, -1, -1) == gs.STATUS_NOT_INITIALIZED
    assert L.gs_gemm_ex_colsplit_multi(None, 0, 0, 4, 4, 4, ctypes.byref(one), ptrs, gs.R_16F, 4, ptrs, gs.R_16F, 4,
                                       ctypes.byref(one), ptrs, gs.R_32F, 4, gs.COMPUTE_32F, -1, -1) \
        == gs.STATUS_NOT_INITIALIZED
    assert L.gs_gemm_batched_ex_multi(None, 0, 0, 4, 4, 4, ctypes.byref(one), ptrs, gs.R_16F, 4, ptrs, gs.R_16F, 4,
                                      ctypes.byref(one), ptrs, gs.R_32F, 4, 2, gs.COMPUTE_32F, -1) \
        == gs.STATUS_NOT_INITIALIZED


@pytest.mark.skipif(gpu_available(), reason="checks behaviour without a GPU")
def test_multi_create_without_gpu_fails_cleanly():
    with pytest.raises(gs.GemmError) as ei:
        gs.MultiHandle([0])
    assert ei.value.status == gs.STATUS_NOT_INITIALIZED
