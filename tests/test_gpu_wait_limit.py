"""The bounded waits of the tensor-core kernel, exercised on purpose.

Every mbarrier wait in k_gemm_tc gives up after the handle's wait limit
(gs_set_wait_limit), records bit 0 and a site code in the device error word and
ends the kernel early, draining what it issued and freeing its tensor memory:
the bounded counterpart of the reference's fence wait with no time limit
(src/vulkan_runner.zig:2197). Here the producer leaves one stage unfilled
(gs_debug_skip_kblock: no expect_tx, no copy, nothing issued after it), so the
MMA issuer's and the epilogue's waits run out after a short limit (2e6 SM cycles,
about a millisecond). The tests check that the call returns, that
gs_device_error reports the timeout and where it happened, and that a call on a
fresh handle right after it is correct against the oracle. No load is left in
flight and nothing faults: this is a wait that ends, not a hang.
"""
import numpy as np
import pytest

import gemm_sm100 as gs
import oracle as orc
from gpu_util import COMPUTE, OUT_OF, assert_parity, make_c, make_input, to_dev, to_host

pytestmark = pytest.mark.gpu

SHORT_LIMIT = 2_000_000  # SM cycles


def _problem(dt, m, n, k, seed):
    rng = np.random.default_rng(seed)
    a, b = make_input(rng, m * k, dt), make_input(rng, k * n, dt)
    c = make_c(rng, m * n, OUT_OF[dt])
    return a, b, c


def _gemm(h, dt, m, n, k, a, b, c, algo):
    dc = to_dev(c)
    h.gemm_ex(0, 0, m, n, k, 1, to_dev(a), dt, m, to_dev(b), dt, k, 0, dc, OUT_OF[dt], m, COMPUTE[dt], algo=algo)
    return dc


def _oracle(dt, m, n, k, a, b, c):
    ref = c.copy()
    assert orc.gemm_ex(0, 0, m, n, k, 1.0, a, dt, m, b, dt, k, 0.0, ref, OUT_OF[dt], m, compute_type=COMPUTE[dt],
                       threads=8) == orc.OK
    return ref


@pytest.mark.parametrize("algo", [0, 1, 2], ids=["tile128x256", "pair256x256", "wide256x512"])
@pytest.mark.parametrize("dt", [gs.R_16F, gs.R_8I])
def test_wait_that_runs_out_ends_the_kernel_and_is_reported(cuda, dt, algo):
    m, n, k = 256, 512, 512
    a, b, c = _problem(dt, m, n, k, 7 + dt + algo)
    with gs.Handle() as h:
        h.set_wait_limit(SHORT_LIMIT)
        h.debug_skip_kblock(2)
        _gemm(h, dt, m, n, k, a, b, c, algo)
        word = h.device_error()  # synchronises: the kernel has ended
    assert word & 1, f"no timeout recorded (word {word:#x})"
    assert (word >> 8) & 0xFF in (3, 4), f"unexpected wait site in {word:#x}"
    # the context is still usable: a fresh handle computes the same problem correctly
    with gs.Handle() as h2:
        got = to_host(_gemm(h2, dt, m, n, k, a, b, c, algo))
        assert h2.device_error() == 0
    assert_parity(got, _oracle(dt, m, n, k, a, b, c), OUT_OF[dt], dt if dt != gs.R_8I else gs.R_32F)


@pytest.mark.parametrize("algo", [0, 1, 2], ids=["tile128x256", "pair256x256", "wide256x512"])
def test_short_wait_limit_does_not_cut_a_healthy_pipeline(cuda, algo):
    dt, m, n, k = gs.R_16F, 512, 1024, 1024
    a, b, c = _problem(dt, m, n, k, 21 + algo)
    with gs.Handle() as h:
        h.set_wait_limit(SHORT_LIMIT)
        got = to_host(_gemm(h, dt, m, n, k, a, b, c, algo))
        assert h.device_error() == 0
    assert_parity(got, _oracle(dt, m, n, k, a, b, c), OUT_OF[dt], dt)


def test_wait_limit_and_hook_arguments(cuda):
    with gs.Handle() as h:
        h.set_wait_limit(0)          # restores the default
        h.debug_skip_kblock(-1)      # off
        with pytest.raises(gs.GemmError):
            h.debug_skip_kblock(-2)
