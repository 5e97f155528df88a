"""GPU tests of the single-process multi-GPU C entry points
(gs_gemm_strided_batched_ex_multi, gs_gemm_batched_ex_multi,
gs_gemm_ex_colsplit_multi) over every visible GPU, and over one GPU.

Each device computes its shard with the same kernel and the same K order as
the single-GPU call, so its part of C must equal the single-GPU result bit for
bit. Gathered C (NCCL point to point) must equal it everywhere it was gathered.
Both the single-GPU result and every gathered C are also compared with the CPU
oracle (the reference's gemmExCuda, src/gemm.zig:671-706) on the same bytes:
bit-exact for INT8 -> INT32, normwise relative error within the FP16 / BF16
bounds otherwise.
"""
import numpy as np
import pytest
import torch

import gemm_sm100 as gs
import oracle as orc
from gpu_util import assert_parity

pytestmark = pytest.mark.gpu

TORCH_OF = {gs.R_16F: torch.float16, gs.R_16BF: torch.bfloat16, gs.R_8I: torch.int8, gs.R_32F: torch.float32,
            gs.R_32I: torch.int32}


def device_sets():
    n = torch.cuda.device_count()
    sets = [[0]]
    if n > 1:
        sets.append(list(range(n)))
    return sets


def _inputs(dt, count, seed):
    g = torch.Generator().manual_seed(seed)
    if dt == gs.R_8I:
        return torch.randint(-128, 128, (count,), generator=g, dtype=torch.int8)
    return (torch.randn(count, generator=g) * 0.25).to(TORCH_OF[dt])


def _np(t):
    """Host bytes of a CPU tensor as the oracle reads them (16-bit floats as raw uint16 bits)."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _oracle(dt, ct, comp, ta, tb, m, n, k, batch, lda, ldb, ldc, sa, sb, sc, A, B, beta, C0) -> np.ndarray:
    c = _np(C0).copy()
    assert orc.gemm_ex(ta, tb, m, n, k, 1.0, _np(A), dt, lda, _np(B), dt, ldb, beta, c, ct, ldc, compute_type=comp,
                       batch=batch, sa=sa, sb=sb, sc=sc, threads=8) == orc.OK
    return c


def _check_oracle(got, want, dt, ct):
    assert_parity(_np(got), want, ct, dt if dt != gs.R_8I else gs.R_32F)


def _ref_strided(dt, ct, comp, ta, tb, m, n, k, batch, lda, ldb, ldc, sa, sb, sc, A, B, beta, C0):
    """(single-GPU result, oracle result); the first is checked against the second here."""
    h = gs.Handle()
    Ad, Bd, Cd = A.cuda(0), B.cuda(0), C0.clone().cuda(0)
    h.gemm_strided_batched_ex(ta, tb, m, n, k, 1, Ad, dt, lda, sa, Bd, dt, ldb, sb, beta, Cd, ct, ldc, sc, batch,
                              comp)
    torch.cuda.synchronize(0)
    out = Cd.cpu()
    want = _oracle(dt, ct, comp, ta, tb, m, n, k, batch, lda, ldb, ldc, sa, sb, sc, A, B, beta, C0)
    _check_oracle(out, want, dt, ct)
    return out, want


@pytest.mark.parametrize("devs", device_sets(), ids=lambda d: f"gpus{len(d)}")
@pytest.mark.parametrize("dt,ta,tb,m,n,k,batch,beta", [
    (gs.R_16F, 0, 0, 256, 384, 512, 12, 0.0),
    (gs.R_8I, 1, 0, 128, 256, 256, 7, 1.0),
    (gs.R_16BF, 0, 1, 200, 136, 96, 5, 0.5),     # ragged edges
])
@pytest.mark.parametrize("gather", [gs.GATHER_NONE, 0, gs.GATHER_ALL])
def test_strided_batched_multi(devs, dt, ta, tb, m, n, k, batch, beta, gather):
    ct = gs.R_32I if dt == gs.R_8I else gs.R_32F
    comp = gs.COMPUTE_32I if dt == gs.R_8I else gs.COMPUTE_32F
    lda, ldb, ldc = (m if ta == 0 else k), (k if tb == 0 else n), m
    sa, sb, sc = m * k, k * n, m * n
    A, B = _inputs(dt, sa * batch, 1), _inputs(dt, sb * batch, 2)
    C0 = (torch.randint(-50, 50, (sc * batch,), dtype=torch.int32) if ct == gs.R_32I
          else torch.randn(sc * batch, dtype=torch.float32))
    ref, want = _ref_strided(dt, ct, comp, ta, tb, m, n, k, batch, lda, ldb, ldc, sa, sb, sc, A, B, beta, C0)

    mh = gs.MultiHandle(devs)
    As = [A.cuda(d) for d in devs]
    Bs = [B.cuda(d) for d in devs]
    Cs = [C0.clone().cuda(d) for d in devs]
    mh.gemm_strided_batched_ex(ta, tb, m, n, k, 1, As, dt, lda, sa, Bs, dt, ldb, sb, beta, Cs, ct, ldc, sc, batch,
                               comp, gather_to=gather)
    off = gs.plan_shards(batch, len(devs), 1)
    gemm_ms, total_ms = mh.last_times()
    for g, d in enumerate(devs):
        got = Cs[g].cpu()
        lo, hi = off[g] * sc, off[g + 1] * sc
        assert torch.equal(got[lo:hi], ref[lo:hi]), f"device {d} shard differs"
        if gather == gs.GATHER_ALL or (gather == g) or len(devs) == 1:
            assert torch.equal(got, ref), f"device {d} gathered C differs"
            _check_oracle(got, want, dt, ct)
        elif gather == gs.GATHER_NONE:
            rest = torch.ones(got.numel(), dtype=torch.bool)
            rest[lo:hi] = False
            assert torch.equal(got[rest], C0[rest]), f"device {d} wrote outside its shard"
        if off[g + 1] > off[g]:
            assert gemm_ms[g] > 0 and total_ms[g] >= gemm_ms[g]
    mh.close()


@pytest.mark.parametrize("devs", device_sets(), ids=lambda d: f"gpus{len(d)}")
@pytest.mark.parametrize("dt,ta,tb,m,n,k", [
    (gs.R_8I, 0, 0, 512, 1280, 256),
    (gs.R_16F, 0, 1, 384, 2048, 320),
    (gs.R_16BF, 1, 0, 256, 1000, 128),           # last block ragged
])
@pytest.mark.parametrize("gather", [gs.GATHER_NONE, 0])
def test_colsplit_multi(devs, dt, ta, tb, m, n, k, gather):
    ct = gs.R_32I if dt == gs.R_8I else gs.R_32F
    comp = gs.COMPUTE_32I if dt == gs.R_8I else gs.COMPUTE_32F
    lda, ldb, ldc = (m if ta == 0 else k), (k if tb == 0 else n), m
    A, B = _inputs(dt, m * k, 3), _inputs(dt, k * n, 4)
    C0 = torch.zeros(m * n, dtype=TORCH_OF[ct])
    ref, want = _ref_strided(dt, ct, comp, ta, tb, m, n, k, 1, lda, ldb, ldc, 0, 0, 0, A, B, 0.0, C0)
    mh = gs.MultiHandle(devs)
    As = [A.cuda(d) for d in devs]
    Bs = [B.cuda(d) for d in devs]
    Cs = [C0.clone().cuda(d) for d in devs]
    mh.gemm_ex_colsplit(ta, tb, m, n, k, 1, As, dt, lda, Bs, dt, ldb, 0, Cs, ct, ldc, comp, gather_to=gather)
    off = gs.plan_shards(n, len(devs), gs.COLSPLIT_ALIGN)
    for g, d in enumerate(devs):
        got = Cs[g].cpu()
        lo, hi = off[g] * ldc, off[g + 1] * ldc
        assert torch.equal(got[lo:hi], ref[lo:hi]), f"device {d} column block differs"
        if gather == g or len(devs) == 1:
            assert torch.equal(got, ref)
            _check_oracle(got, want, dt, ct)
    mh.close()


@pytest.mark.parametrize("devs", device_sets(), ids=lambda d: f"gpus{len(d)}")
def test_pointer_array_multi(devs):
    dt, ct, comp = gs.R_16F, gs.R_32F, gs.COMPUTE_32F
    m, n, k, batch = 128, 256, 192, 9
    mats_a = [_inputs(dt, m * k, 10 + i) for i in range(batch)]
    mats_b = [_inputs(dt, k * n, 40 + i) for i in range(batch)]
    A = torch.cat(mats_a)
    B = torch.cat(mats_b)
    ref, want = _ref_strided(dt, ct, comp, 0, 0, m, n, k, batch, m, k, m, m * k, k * n, m * n, A, B, 0.0,
                             torch.zeros(m * n * batch))
    mh = gs.MultiHandle(devs)
    keep, arrs = [], ([], [], [])
    for d in devs:
        # scattered per-entry buffers on each device
        a_list = [x.cuda(d) for x in mats_a]
        b_list = [x.cuda(d) for x in mats_b]
        c_list = [torch.zeros(m * n, dtype=torch.float32, device=f"cuda:{d}") for _ in range(batch)]
        keep.append((a_list, b_list, c_list))
        for arr, lst in zip(arrs, (a_list, b_list, c_list)):
            arr.append(torch.tensor([t.data_ptr() for t in lst], dtype=torch.int64, device=f"cuda:{d}"))
    mh.gemm_batched_ex(0, 0, m, n, k, 1, arrs[0], dt, m, arrs[1], dt, k, 0, arrs[2], ct, m, batch, comp)
    off = gs.plan_shards(batch, len(devs), 1)
    for g, d in enumerate(devs):
        c_list = keep[g][2]
        for i in range(batch):
            got = c_list[i].cpu()
            if off[g] <= i < off[g + 1]:
                assert torch.equal(got, ref[i * m * n:(i + 1) * m * n]), f"device {d} entry {i}"
                _check_oracle(got, want[i * m * n:(i + 1) * m * n], dt, ct)
            else:
                assert not got.any(), f"device {d} wrote entry {i} outside its shard"
    mh.close()


def test_gather_needs_dense_c():
    devs = list(range(torch.cuda.device_count()))
    if len(devs) < 2:
        devs = [0]
    mh = gs.MultiHandle(devs)
    m, n, k = 128, 256, 64
    A = [torch.zeros(m * k, dtype=torch.float16, device=f"cuda:{d}") for d in devs]
    B = [torch.zeros(k * n, dtype=torch.float16, device=f"cuda:{d}") for d in devs]
    C = [torch.zeros((m + 8) * n, dtype=torch.float32, device=f"cuda:{d}") for d in devs]
    s = mh.gemm_ex_colsplit(0, 0, m, n, k, 1, A, gs.R_16F, m, B, gs.R_16F, k, 0, C, gs.R_32F, m + 8,
                            gs.COMPUTE_32F, gather_to=0, check=False)
    assert s == (gs.STATUS_NOT_SUPPORTED if len(devs) > 1 else gs.STATUS_SUCCESS)
    s = mh.gemm_ex_colsplit(0, 0, m, n, k, 1, A, gs.R_16F, m, B, gs.R_16F, k, 0, C, gs.R_32F, m + 8,
                            gs.COMPUTE_32F, gather_to=len(devs), check=False)
    assert s == gs.STATUS_INVALID_VALUE
    # an invalid problem is rejected before any launch
    s = mh.gemm_ex_colsplit(0, 0, m, n, k, 1, A, gs.R_16F, m - 1, B, gs.R_16F, k, 0, C, gs.R_32F, m,
                            gs.COMPUTE_32F, check=False)
    assert s == gs.STATUS_INVALID_VALUE
    mh.close()
