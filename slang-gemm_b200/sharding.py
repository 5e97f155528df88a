"""Multi-GPU sharding of the GEMM call family: one process per GPU.

Neither split needs a reduction:
  * batched calls (gemmStridedBatchedEx / gemmBatchedEx) split by batch entry:
    rank g computes entries [cut[g], cut[g+1]);
  * one large GEMM splits by column blocks of B and C: rank g holds all of A
    and computes C[:, cut[g]:cut[g+1]]. In column-major storage a column block
    of C is one contiguous range, so per-rank blocks concatenate into C.
The cut points come from the library's gs_plan_shards. The only collectives
are the optional all-gather that assembles C on every rank (for callers that
want it on one device) and a status all-reduce before it, so that a rank whose
compute failed makes every rank raise instead of leaving the others waiting in
the gather. A rank that dies outright is reported by the process group's own
timeout on the next collective.
"""
from __future__ import annotations

from dataclasses import dataclass

import gemm_sm100 as gs


class ShardFailed(RuntimeError):
    """Raised on every rank when at least one rank's local compute failed."""


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    kind: str      # "cols" or "batch"
    begin: int     # first unit (column or batch entry) of this rank
    end: int       # one past the last unit
    cuts: tuple    # all world+1 cut points

    @property
    def size(self) -> int:
        return self.end - self.begin


def plan(units: int, world: int, rank: int, kind: str, align: int = 1) -> Shard:
    """This rank's share of `units` columns ("cols") or batch entries ("batch")."""
    if kind not in ("cols", "batch"):
        raise ValueError(kind)
    cuts = gs.plan_shards(units, world, align)
    return Shard(rank, world, kind, cuts[rank], cuts[rank + 1], tuple(cuts))


@dataclass(frozen=True)
class LocalProblem:
    """Element offsets into the caller's full A, B, C and the local shape."""
    a_off: int
    b_off: int
    c_off: int
    n: int
    batch: int


def local_problem(s: Shard, n: int, batch: int, trans_b: int, ldb: int, ldc: int, stride_a: int = 0,
                  stride_b: int = 0, stride_c: int = 0) -> LocalProblem:
    """Offsets (in elements) of this rank's operands inside the full column-major buffers.

    cols: B op N is k x n (column j at j*ldb), B op T is stored n x k (row j at j);
          C column j at j*ldc; A is used whole.
    batch: every operand advances by its batch stride.
    """
    if s.kind == "cols":
        b_off = s.begin if trans_b else s.begin * ldb
        return LocalProblem(0, b_off, s.begin * ldc, s.size, batch)
    return LocalProblem(s.begin * stride_a, s.begin * stride_b, s.begin * stride_c, n, s.size)


def check_all_ok(ok: bool, group=None) -> None:
    """Status all-reduce: every rank learns whether any rank failed before the data collective."""
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    if int(flag.item()) != 0:
        raise ShardFailed("a rank's local GEMM failed; no rank entered the gather")


def gather_blocks(local, s: Shard, unit_elems: int, group=None):
    """All-gather the per-rank contiguous blocks (`s.size * unit_elems` elements each) into the
    full buffer on every rank. Unequal blocks are padded to the largest for the collective."""
    import torch
    import torch.distributed as dist

    sizes = [(s.cuts[g + 1] - s.cuts[g]) * unit_elems for g in range(s.world)]
    width = max(sizes) if sizes else 0
    send = torch.zeros(width, dtype=local.dtype, device=local.device)
    send[: local.numel()] = local.reshape(-1)
    recv = torch.empty(width * s.world, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    parts = [recv[g * width: g * width + sizes[g]] for g in range(s.world)]
    return torch.cat(parts)


def run_sharded(compute, s: Shard, local_c, unit_elems: int, gather: bool = True, group=None):
    """Runs `compute()` (this rank's GEMM into local_c), propagates failures to every rank,
    then optionally assembles C on every rank. Returns the full C (gather) or local_c."""
    ok = True
    err = None
    try:
        compute()
    except Exception as e:  # reported to all ranks below, re-raised here
        ok = False
        err = e
    try:
        check_all_ok(ok, group)
    except ShardFailed:
        if err is not None:
            raise ShardFailed(f"rank {s.rank}: {err}") from err
        raise
    if not gather:
        return local_c
    return gather_blocks(local_c, s, unit_elems, group)
