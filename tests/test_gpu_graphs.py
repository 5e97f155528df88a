"""The device entry points inside CUDA graphs: after one warm-up call (which
sets kernel attributes and allocates the handle's tensor-map buffer), a call
captured into a graph and replayed must give the same bits as the direct
call, for every kernel family (tensor-core single / strided / pointer-array / split-K,
FFMA data-parallel and stream-K, the FAST_TF32 split + tf32 GEMM, CUDA-core
fallback, k = 0)."""
import numpy as np
import pytest
import torch

import gemm_sm100 as gs
from gpu_util import COMPUTE, OUT_OF, make_input

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("dt,m,n,k,batch,lda_pad,ptr,algo", [
    (gs.R_16F, 512, 768, 256, 1, 0, False, -1),     # tensor core, wide tile
    (gs.R_16BF, 384, 256, 192, 3, 0, False, 1),     # tensor core, strided batch, pair tile
    (gs.R_8I, 256, 512, 256, 4, 0, True, -1),       # tensor core, pointer-array batch (map builder + GEMM)
    (gs.R_32F, 300, 200, 100, 2, 0, False, -1),     # FFMA sgemm
    (gs.R_16F, 100, 60, 40, 1, 3, False, -1),       # CUDA-core fallback (misaligned leading dimension)
    (gs.R_16F, 64, 64, 0, 1, 0, False, -1),         # k == 0: beta only
    (gs.R_32F, 1024, 512, 1100, 1, 0, False, -1),   # FAST_TF32: split kernels + chunked kind::tf32 GEMM
    (gs.R_32F, 1600, 1100, 1030, 2, 0, False, -1),  # FFMA stream-K (234 tiles on 296 slots): workspace, counters
    (gs.R_16F, 512, 512, 16384, 1, 0, False, -1),   # tensor-core split-K: 16 slices into a workspace + reduction
])
def test_graph_replay_matches_direct_call(dt, m, n, k, batch, lda_pad, ptr, algo):
    rng = np.random.default_rng(m + n + k)
    ct, comp = OUT_OF[dt], COMPUTE[dt]
    lda, ldb, ldc = m + lda_pad, max(k, 1), m
    sa, sb, sc = lda * max(k, 1), ldb * n, ldc * n
    A = _dev(make_input(rng, sa * batch, dt))
    B = _dev(make_input(rng, sb * batch, dt))
    C0 = torch.from_numpy(rng.integers(-5, 5, sc * batch).astype(np.int32 if ct == gs.R_32I else np.float32)).cuda()
    alpha, beta = (2.0, 1.0) if dt == gs.R_8I else (1.5, 0.5)
    stream = torch.cuda.Stream()
    h = gs.Handle(stream)
    es = A.element_size()
    ec = C0.element_size()

    def call(C):
        if ptr:
            arr = lambda t, s, e: torch.tensor([t.data_ptr() + j * s * e for j in range(batch)],  # noqa
                                               dtype=torch.int64, device="cuda")
            return h.gemm_batched_ex(0, 0, m, n, k, alpha, arr(A, sa, es), dt, lda, arr(B, sb, es), dt, ldb, beta,
                                     arr(C, sc, ec), ct, ldc, batch, comp, algo=algo)
        if dt == gs.R_32F and batch == 1 and k > 1000:
            return h.gemm_ex(0, 0, m, n, k, alpha, A, dt, lda, B, dt, ldb, beta, C, ct, ldc,
                             gs.COMPUTE_32F_FAST_TF32)
        if dt == gs.R_32F and batch == 1:
            return h.sgemm(0, 0, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
        return h.gemm_strided_batched_ex(0, 0, m, n, k, alpha, A, dt, lda, sa, B, dt, ldb, sb, beta, C, ct, ldc, sc,
                                         batch, comp, algo=algo)

    direct = C0.clone()
    with torch.cuda.stream(stream):
        call(direct)                                   # warm-up: attributes, tensor-map buffer, workspaces
    stream.synchronize()
    captured = C0.clone()
    if ptr:
        # pointer arrays must exist before capture (their contents are read at replay)
        arrs = [torch.tensor([t.data_ptr() + j * s * e for j in range(batch)], dtype=torch.int64, device="cuda")
                for t, s, e in ((A, sa, es), (B, sb, es), (captured, sc, ec))]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        if ptr:
            h.gemm_batched_ex(0, 0, m, n, k, alpha, arrs[0], dt, lda, arrs[1], dt, ldb, beta, arrs[2], ct, ldc,
                              batch, comp, algo=algo)
        else:
            call(captured)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, direct)
    # replaying again applies the GEMM again on top (beta != 0): same as a second direct call. The replay
    # goes on the handle's stream, ordered before the direct call: both use the handle's workspaces.
    with torch.cuda.stream(stream):
        g.replay()
        call(direct)
    torch.cuda.synchronize()
    assert torch.equal(captured, direct)
    assert h.device_error() == 0
    del g
