"""GPU test of gs_gemm_batched_ex_noalloc, the pointer-array batched GEMM for
callers that cannot allocate device memory (their memory belongs to a
framework's caching allocator or a fixed budget, or they must not pay the
synchronisation cudaMalloc/cudaFree can imply).

It checks, through the C ABI, that the no-allocation entry point produces the
same C as the regular entry point gs_gemm_batched_ex on the same inputs, on two
calls in a row (the second call reuses the static scratch the first one left
behind), within the tolerances the other parity tests use: bit-exact for
INT8 -> INT32, normwise relative error <= 2e-3 for FP16 and <= 1e-2 for BF16.
This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
from gpu_util import COMPUTE, NP_OF, OUT_OF, assert_parity, make_c, make_input, to_dev, to_host

pytestmark = pytest.mark.gpu


def _batch(rng, dt, m, n, k, batch, shift=0):
    import torch

    ct = OUT_OF[dt]
    es = np.dtype(NP_OF[dt]).itemsize
    a = [to_dev(make_input(rng, m * k + 16, dt)) for _ in range(batch)]
    b = [to_dev(make_input(rng, k * n, dt)) for _ in range(batch)]
    c0 = [make_c(rng, m * n, ct) for _ in range(batch)]
    ptrs = lambda ts, off=0: torch.tensor([t.data_ptr() + off for t in ts], dtype=torch.int64, device="cuda")  # noqa
    return a, b, c0, ptrs(a, shift * es), ptrs(b)


@pytest.mark.parametrize("dt,shift", [(gs.R_16F, 0), (gs.R_16BF, 0), (gs.R_8I, 0), (gs.R_16F, 1)])
def test_noalloc_matches_regular_entry_point_twice(cuda, dt, shift):
    import torch

    ct = OUT_OF[dt]
    comp = COMPUTE[dt]
    m, n, k, batch = 272, 264, 192, 6
    alpha, beta = (2.0, -1.0) if dt == gs.R_8I else (0.75, 0.5)
    stream = torch.cuda.current_stream()
    with gs.Handle(stream=stream) as h:
        for call in range(2):  # two calls in a row on the shared static scratch
            rng = np.random.default_rng(100 + 10 * call + dt)
            a, b, c0, aptr, bptr = _batch(rng, dt, m, n, k, batch, shift)
            c_reg = [to_dev(x) for x in c0]
            c_na = [to_dev(x) for x in c0]
            creg = torch.tensor([t.data_ptr() for t in c_reg], dtype=torch.int64, device="cuda")
            cna = torch.tensor([t.data_ptr() for t in c_na], dtype=torch.int64, device="cuda")
            h.gemm_batched_ex(0, 0, m, n, k, alpha, aptr, dt, m, bptr, dt, k, beta, creg, ct, m, batch, comp)
            s = gs.gemm_batched_ex_noalloc(stream, 0, 0, m, n, k, alpha, aptr, dt, m, bptr, dt, k, beta, cna, ct,
                                           m, batch, comp)
            assert s == gs.STATUS_SUCCESS, gs.status_name(s)
            torch.cuda.synchronize()
            for i in range(batch):
                assert_parity(to_host(c_na[i]), to_host(c_reg[i]), ct, dt if dt != gs.R_8I else gs.R_32F)
                assert not np.array_equal(to_host(c_na[i]), c0[i]), "no-allocation call left C untouched"


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    import torch

    dummy = torch.zeros(64, dtype=torch.int64, device="cuda")
    s = gs.gemm_batched_ex_noalloc(None, 0, 0, 16, 16, 16, 1.0, dummy, gs.R_16F, 16, dummy, gs.R_16F, 16, 0.0,
                                   dummy, gs.R_32F, 16, gs.NOALLOC_MAX_BATCH + 1, gs.COMPUTE_32F)
    assert s == gs.STATUS_INVALID_VALUE
