"""Multi-rank host logic of the sharded GEMM, on CPU with world-size-2 gloo.

Each rank computes its shard with the CPU oracle (the stand-in for its GPU's
kernel), the shards are assembled with the all-gather of sharding.py, and the
result must equal the oracle's full result bit for bit (same per-element
arithmetic). Failure handling: a rank whose compute raises makes every rank
raise ShardFailed (nobody waits in the gather); a rank that exits before the
collective makes the survivor's collective fail within the process group's
timeout.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PATHS = [os.path.join(ROOT, "slang-gemm_b200"), os.path.join(ROOT, "oracle"), HERE]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    import datetime

    import torch.distributed as dist

    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _inputs(kind):
    import oracle as orc

    rng = np.random.default_rng(7)
    if kind == "cols":
        m, n, k, batch = 48, 40, 24, 1
    else:
        m, n, k, batch = 24, 20, 16, 5
    a = orc.randn_lowp(rng, m * k * batch, orc.R_16F)
    b = orc.randn_lowp(rng, k * n * batch, orc.R_16F)
    c = np.zeros(m * n * batch, np.float32)
    return m, n, k, batch, a, b, c


def _worker(rank, world, port, kind, trans_b, out_q):
    dist = _init(rank, world, port)
    try:
        import oracle as orc
        import sharding

        m, n, k, batch, a, b, c = _inputs(kind)
        ldb = n if trans_b else k
        units = n if kind == "cols" else batch
        s = sharding.plan(units, world, rank, kind, align=8 if kind == "cols" else 1)
        lp = sharding.local_problem(s, n, batch, trans_b, ldb, m, m * k, k * n, m * n)
        local_c = np.zeros(m * lp.n * lp.batch, np.float32)

        def compute():
            rc = orc.gemm_ex(0, trans_b, m, lp.n, k, 1.0, a[lp.a_off:], orc.R_16F, m, b[lp.b_off:], orc.R_16F, ldb,
                             0.0, local_c, orc.R_32F, m, batch=lp.batch, sa=m * k, sb=k * n, sc=m * lp.n)
            assert rc == orc.OK

        unit = m if kind == "cols" else m * n
        full = sharding.run_sharded(compute, s, torch.from_numpy(local_c), unit, gather=True)
        ref = c.copy()
        assert orc.gemm_ex(0, trans_b, m, n, k, 1.0, a, orc.R_16F, m, b, orc.R_16F, ldb, 0.0, ref, orc.R_32F, m,
                           batch=batch, sa=m * k, sb=k * n, sc=m * n) == orc.OK
        out_q.put((rank, bool(np.array_equal(full.numpy().view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


def _spawn(fn, args, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = []
    while not q.empty():
        results.append(q.get())
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    return sorted(results), codes


@pytest.mark.parametrize("kind,trans_b", [("cols", 0), ("cols", 1), ("batch", 0)])
def test_sharded_gemm_equals_full_oracle(kind, trans_b):
    results, codes = _spawn(_worker, (kind, trans_b))
    assert codes == [0, 0], codes
    assert results == [(0, True), (1, True)], results


def _failing_worker(rank, world, port, out_q):
    dist = _init(rank, world, port)
    try:
        import sharding

        s = sharding.plan(16, world, rank, "batch")

        def compute():
            if rank == 1:
                raise RuntimeError("injected failure on the host")

        try:
            sharding.run_sharded(compute, s, torch.zeros(s.size * 4), 4, gather=True)
            out_q.put((rank, "no error"))
        except sharding.ShardFailed:
            out_q.put((rank, "ShardFailed"))
    finally:
        dist.destroy_process_group()


def test_failed_rank_makes_every_rank_raise():
    results, codes = _spawn(_failing_worker, ())
    assert codes == [0, 0], codes
    assert results == [(0, "ShardFailed"), (1, "ShardFailed")], results


def _vanishing_worker(rank, world, port, out_q):
    dist = _init(rank, world, port, timeout_s=5)
    import sharding

    s = sharding.plan(16, world, rank, "batch")
    if rank == 1:
        os._exit(0)  # leaves between steps, no collective in flight
    try:
        sharding.run_sharded(lambda: None, s, torch.zeros(s.size * 4), 4, gather=True)
        out_q.put((rank, "no error"))
    except Exception as e:  # gloo reports the missing peer (timeout or closed connection)
        out_q.put((rank, type(e).__name__))


def test_vanished_rank_is_detected_by_collective_timeout():
    results, codes = _spawn(_vanishing_worker, ())
    assert results and results[0][0] == 0 and results[0][1] != "no error", results
