"""GPU tests of gs_gemm_batched_ex_noalloc, the pointer-array batched GEMM for
callers that cannot allocate device memory: a framework whose caching allocator
owns the GPU's memory, a service that plans a fixed memory budget up front, or
a latency-critical path that must not pay the device-wide synchronisation
cudaMalloc/cudaFree can imply. Its scratch is a static device array, so it needs
no handle and no allocation.

Through the C ABI, on two calls in a row (the second reuses the static scratch
the first one left behind), each case checks the no-allocation result against
the regular entry point gs_gemm_batched_ex on the same inputs and against the
CPU oracle's restatement of the reference's gemmBatchedEx
(src/gemm.zig:636-663), within the tolerances of the other parity tests:
bit-exact for INT8 -> INT32, normwise relative error <= 1e-5 (FP32), 2e-3
(FP16), 1e-2 (BF16). Cases cover every route the entry point takes: the
tensor-core kernel with per-entry tensor maps (beta != 0, and beta == 0 where C
goes out through per-entry TMA-store maps, with and without a misaligned C
entry), the FFMA kernel (FP32), the CUDA-core kernel (a leading dimension TMA
cannot address), k == 0 (C = beta * C) and a batch of exactly
GS_NOALLOC_MAX_BATCH. After each call gs_noalloc_device_error must read 0.
This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import COMPUTE, NP_OF, OUT_OF, assert_parity, make_c, make_input, to_dev, to_host

pytestmark = pytest.mark.gpu

# name -> (dt, m, n, k, batch, lda_pad, shift_a, alpha, beta, c_shift_entry)
CASES = {
    "f16-beta": (gs.R_16F, 272, 264, 192, 6, 0, 0, 0.75, 0.5, -1),
    "bf16-beta": (gs.R_16BF, 272, 264, 192, 6, 0, 0, 0.75, 0.5, -1),
    "i8-beta": (gs.R_8I, 272, 264, 192, 6, 0, 0, 2.0, -1.0, -1),
    "f16-misaligned-a": (gs.R_16F, 272, 264, 192, 6, 0, 1, 0.75, 0.5, -1),
    "f16-beta0-tma-store": (gs.R_16F, 300, 136, 96, 4, 0, 0, 1.0, 0.0, -1),
    "i8-beta0-tma-store": (gs.R_8I, 300, 136, 96, 4, 0, 0, 1.0, 0.0, -1),
    "f16-beta0-misaligned-c": (gs.R_16F, 300, 136, 96, 4, 0, 0, 1.0, 0.0, 2),
    "f32-ffma": (gs.R_32F, 200, 150, 96, 5, 0, 0, 1.5, 0.5, -1),
    "f16-odd-lda-simt": (gs.R_16F, 130, 70, 66, 3, 3, 0, 0.75, 0.5, -1),
    "f16-k0": (gs.R_16F, 96, 80, 0, 3, 0, 0, 0.75, 0.5, -1),
    "f16-max-batch": (gs.R_16F, 64, 64, 64, gs.NOALLOC_MAX_BATCH, 0, 0, 1.0, 0.0, -1),
}


def _run_case(rng, dt, m, n, k, batch, lda_pad, shift, alpha, beta, c_shift_entry):
    import torch

    ct = OUT_OF[dt]
    comp = COMPUTE[dt]
    es, ec = np.dtype(NP_OF[dt]).itemsize, np.dtype(NP_OF[ct]).itemsize
    lda = m + lda_pad
    a = [make_input(rng, lda * max(k, 1) + 16, dt) for _ in range(batch)]
    b = [make_input(rng, max(k, 1) * n, dt) for _ in range(batch)]
    c0 = [make_c(rng, m * n + 8, ct) for _ in range(batch)]
    da, db = [to_dev(x) for x in a], [to_dev(x) for x in b]
    c_reg, c_na = [to_dev(x) for x in c0], [to_dev(x) for x in c0]

    def ptrs(ts, off=0, entry=-1, entry_off=0):
        return torch.tensor([t.data_ptr() + off + (entry_off if i == entry else 0) for i, t in enumerate(ts)],
                            dtype=torch.int64, device="cuda")

    aptr, bptr = ptrs(da, shift * es), ptrs(db)
    c_off = 1 * ec  # one element: breaks the 16-byte alignment of one C entry
    creg, cna = ptrs(c_reg, 0, c_shift_entry, c_off), ptrs(c_na, 0, c_shift_entry, c_off)
    stream = torch.cuda.current_stream()
    with gs.Handle(stream=stream) as h:
        h.gemm_batched_ex(0, 0, m, n, k, alpha, aptr, dt, lda, bptr, dt, max(k, 1), beta, creg, ct, m, batch, comp)
    s = gs.gemm_batched_ex_noalloc(stream, 0, 0, m, n, k, alpha, aptr, dt, lda, bptr, dt, max(k, 1), beta, cna, ct,
                                   m, batch, comp)
    assert s == gs.STATUS_SUCCESS, gs.status_name(s)
    st, word = gs.noalloc_device_error(stream)
    assert st == gs.STATUS_SUCCESS and word == 0, f"device error word {word:#x}"
    # the oracle on the same bytes: entry i reads A at shift and writes C at its (maybe shifted) start
    a_view = [x[shift:shift + lda * max(k, 1)].copy() for x in a]
    refs = [x.copy() for x in c0]
    views = [r[(1 if i == c_shift_entry else 0):][: m * n] for i, r in enumerate(refs)]
    outs = [v.copy() for v in views]
    assert orc.gemm_batched_ex(0, 0, m, n, k, alpha, a_view, dt, lda, b, dt, max(k, 1), beta, outs, ct, m,
                               compute_type=comp) == orc.OK
    tol_dt = dt if dt != gs.R_8I else gs.R_32F
    for i in range(batch):
        lo = 1 if i == c_shift_entry else 0
        got, reg = to_host(c_na[i]), to_host(c_reg[i])
        assert_parity(got[lo:lo + m * n], outs[i], ct, tol_dt)          # against the oracle
        assert_parity(got[lo:lo + m * n], reg[lo:lo + m * n], ct, tol_dt)  # against gs_gemm_batched_ex
        # bytes outside this entry's C are untouched
        np.testing.assert_array_equal(np.delete(got, np.s_[lo:lo + m * n]), np.delete(c0[i], np.s_[lo:lo + m * n]))


@pytest.mark.parametrize("name", sorted(CASES))
def test_noalloc_matches_oracle_and_regular_entry_point_twice(cuda, name):
    dt, m, n, k, batch, lda_pad, shift, alpha, beta, c_shift = CASES[name]
    for call in range(2):  # two calls in a row on the shared static scratch
        rng = np.random.default_rng(100 + 10 * call + dt + len(name))
        _run_case(rng, dt, m, n, k, batch, lda_pad, shift, alpha, beta, c_shift)


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    import torch

    dummy = torch.zeros(64, dtype=torch.int64, device="cuda")
    s = gs.gemm_batched_ex_noalloc(None, 0, 0, 16, 16, 16, 1.0, dummy, gs.R_16F, 16, dummy, gs.R_16F, 16, 0.0,
                                   dummy, gs.R_32F, 16, gs.NOALLOC_MAX_BATCH + 1, gs.COMPUTE_32F)
    assert s == gs.STATUS_INVALID_VALUE
    st, word = gs.noalloc_device_error(None)
    assert st == gs.STATUS_SUCCESS and word == 0
