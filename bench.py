#!/usr/bin/env python3
"""Benchmark of libgemm_sm100 on the configurations slang-gemm's north star names.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

One step is one call of the hot path over one batch of synthetic input (one
gemmEx / gemmStridedBatchedEx / sgemm). The default workload is configuration
C3 of the north star at the size the headline metric is quoted on:
gemmEx, A and B CUDA_R_16F ~ N(0,1)*0.25, C CUDA_R_32F, CUBLAS_COMPUTE_32F,
op N/N, M = N = K = 8192, alpha = 1, beta = 0.

Rank 0 prints ONE JSON line:
  value     whole-job TFLOP/s (TOP/s for INT8) with inputs resident in HBM,
            device-timed with CUDA events on the launching stream, max over ranks;
  e2e       the same metric through the host-buffer entry point gs_host_gemm_ex
            (pinned host A/B in, C out, copies inside the timed region);
  roofline  the tensor-core kernel against the measured B200 peak;
  cpu_baseline  the C restatement of the reference's scalar gemmEx (oracle/)
            timed on this host's cores on a bounded sample of the same GEMM.
With N > 1 ranks (torchrun, NCCL), the work is sharded with no data-path
collective: column blocks of B and C for single GEMMs, batch entries for
batched calls, each rank holding a fixed share (weak scaling).

`--impl reference` times the reference's own CPU algorithm (the oracle port of
src/gemm.zig gemmExCuda, all host threads) on the same config and metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "slang-gemm_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

METRIC = "gemmEx TFLOPS/TOPS at 8192³ vs B200 dense peak; shader_cublas_ratio"

# name -> workload. dt/ct: CUDA data types; shard: how N > 1 ranks split the work.
CONFIGS = {
    "c3-f16-nn": dict(api="ex", dt=2, ct=0, comp=68, op=(0, 0), m=8192, n=8192, k=8192, batch=1, alpha=1.0, beta=0.0,
                      shard="cols", label="gemmEx C3: A,B CUDA_R_16F N(0,1)*0.25, C CUDA_R_32F, COMPUTE_32F, op N/N, "
                                          "M=N=K=8192, alpha=1, beta=0"),
    "c3-f16-tn": dict(api="ex", dt=2, ct=0, comp=68, op=(1, 0), m=8192, n=8192, k=8192, batch=1, alpha=1.0, beta=0.0,
                      shard="cols", label="gemmEx C3: A,B CUDA_R_16F, C CUDA_R_32F, COMPUTE_32F, op T/N, M=N=K=8192"),
    "c3-bf16-nn": dict(api="ex", dt=14, ct=0, comp=68, op=(0, 0), m=8192, n=8192, k=8192, batch=1, alpha=1.0,
                       beta=0.0, shard="cols",
                       label="gemmEx C3: A,B CUDA_R_16BF, C CUDA_R_32F, COMPUTE_32F, op N/N, M=N=K=8192"),
    "c3-f16-nn-4096": dict(api="ex", dt=2, ct=0, comp=68, op=(0, 0), m=4096, n=4096, k=4096, batch=1, alpha=1.0,
                           beta=0.0, shard="cols", label="gemmEx C3: f16 -> f32, op N/N, M=N=K=4096"),
    "c5-i8-nn": dict(api="ex", dt=3, ct=10, comp=72, op=(0, 0), m=8192, n=8192, k=8192, batch=1, alpha=1.0, beta=0.0,
                     shard="cols", label="gemmEx C5: A,B CUDA_R_8I uniform [-128,127], C CUDA_R_32I, COMPUTE_32I, "
                                         "op N/N, M=N=K=8192, alpha=1, beta=0"),
    "c4-f16-strided": dict(api="strided", dt=2, ct=0, comp=68, op=(0, 0), m=512, n=512, k=1024, batch=256,
                           alpha=1.0 / 32.0, beta=0.0, shard="batch",
                           label="gemmStridedBatchedEx C4: f16 -> f32, batch 256, M=N=512, K=1024, "
                                 "strides MK/KN/MN, alpha=1/sqrt(K), beta=0"),
    "c5b-i8-strided": dict(api="strided", dt=3, ct=10, comp=72, op=(0, 0), m=2048, n=2048, k=2048, batch=64,
                           alpha=1.0, beta=0.0, shard="batch",
                           label="gemmStridedBatchedEx C5b: s8 -> s32, batch 64, M=N=K=2048"),
    "c3-f32-fast-tf32": dict(api="ex", dt=0, ct=0, comp=77, op=(0, 0), m=8192, n=8192, k=8192, batch=1, alpha=1.0,
                             beta=0.0, shard="cols",
                             label="gemmEx: A,B,C CUDA_R_32F uniform [-1,1), COMPUTE_32F_FAST_TF32 (three tf32 "
                                   "products per f32 product, FP32 tolerance), op N/N, M=N=K=8192"),
    "c2-sgemm-nn": dict(api="sgemm", dt=0, ct=0, comp=68, op=(0, 0), m=4096, n=1024, k=2048, batch=1, alpha=1.5,
                        beta=0.5, shard="cols", label="sgemm C2: FP32 op N/N, 4096x1024x2048, alpha=1.5, beta=0.5"),
    "c2-sgemm-tt": dict(api="sgemm", dt=0, ct=0, comp=68, op=(1, 1), m=1024, n=4096, k=512, batch=1, alpha=1.5,
                        beta=0.5, shard="cols", label="sgemm C2: FP32 op T/T, 1024x4096x512, alpha=1.5, beta=0.5"),
    "c1-sgemm-512": dict(api="sgemm", dt=0, ct=0, comp=68, op=(0, 0), m=512, n=512, k=512, batch=1, alpha=1.0,
                         beta=0.0, shard="cols", label="sgemm C1: FP32 op N/N, 512^3, alpha=1, beta=0"),
}
ELEM = {0: 4, 2: 2, 3: 1, 10: 4, 14: 2}
DTYPE_NAME = {0: "f32", 2: "f16", 3: "s8", 14: "bf16"}


# NVIDIA's dense (non-sparse) B200 figures, for context beside the measured denominators:
# FP16/BF16 2.25 PFLOP/s, INT8 4.5 POP/s, TF32 1.125 PFLOP/s, HBM3e 7.7 TB/s (HGX).
DATASHEET = {"tensor16": 2250.0, "tensor8": 4500.0, "tf32": 1125.0, "hbm_gbs": 7700.0}


def load_peaks() -> dict:
    """Roofline denominators: MEASURED_PEAKS.json (driver-written) or the pool's fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "sm_max_mhz": float(d.get("sm_max_mhz", 1965.0)), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "sm_max_mhz": 1965.0,
                "source": "fallback"}


def work(cfg: dict) -> tuple[float, float]:
    """(algorithmic flops, algorithmic bytes) of one step of one rank's share."""
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    es, ec = ELEM[cfg["dt"]], ELEM[cfg["ct"]]
    flops = 2.0 * m * n * k * b
    byts = b * (m * k * es + k * n * es + m * n * ec * (2 if cfg["beta"] != 0 else 1))
    return flops, float(byts)


def roofline_of(cfg: dict, flops: float, byts: float, ms_per_launch: float, peaks: dict, traffic) -> dict:
    """Tensor-core bound for the 8192^3 GEMMs; HBM bound for the batched f16 config; FFMA for sgemm."""
    ai = flops / byts
    if cfg["api"] == "sgemm":
        peak = 148 * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12
        achieved = flops / (ms_per_launch * 1e-3) / 1e12
        return {"bound": "ffma", "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": "nominal 148 SM x 128 FP32 lanes x 2 x max SM clock (no measured FFMA peak)"}
    tsrc = ("profiles/dram_traffic.json: committed ncu capture of this configuration (dram__bytes_read.sum + "
            "dram__bytes_write.sum per launch), not measured in this run") if traffic is not None else None
    if cfg["comp"] == 77:
        # FAST_TF32: the dense tf32 rate is half the bf16 rate; the kernel runs three tf32 products per f32
        # product, so `achieved` (algorithmic 2MNK) can reach at most a third of this peak.
        peak = peaks["bf16"] / 2.0
        achieved = flops / (ms_per_launch * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": tsrc,
                "peak_source": f"{peaks['source']} cuBLAS bf16 burst / 2 (dense tf32); the kernel executes "
                               "3 tf32 products per f32 product, so hardware work is 3x achieved",
                "peak_datasheet": DATASHEET["tf32"], "frac_datasheet": round(achieved / DATASHEET["tf32"], 4)}
    tensor_peak = peaks["bf16"] * (2.0 if cfg["dt"] == 3 else 1.0)
    ridge = tensor_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if ai < ridge:
        achieved = byts / (ms_per_launch * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic, "traffic_source": tsrc,
                "peak_source": f"{peaks['source']} HBM copy bandwidth",
                "peak_datasheet": DATASHEET["hbm_gbs"], "frac_datasheet": round(achieved / DATASHEET["hbm_gbs"], 4)}
    achieved = flops / (ms_per_launch * 1e-3) / 1e12
    src = f"{peaks['source']} cuBLAS bf16 burst" + (" x2 for INT8 (dense INT8 rate is twice BF16 on B200; no "
                                                    "INT8 peak is measured)" if cfg["dt"] == 3 else "")
    sheet = DATASHEET["tensor8"] if cfg["dt"] == 3 else DATASHEET["tensor16"]
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tensor_peak, 1),
            "unit": "TOP/s" if cfg["dt"] == 3 else "TFLOP/s", "frac": round(achieved / tensor_peak, 4),
            "traffic": traffic, "traffic_source": tsrc, "peak_source": src,
            "peak_datasheet": sheet, "frac_datasheet": round(achieved / sheet, 4)}


def committed_traffic(name: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        return json.load(open(p)).get(name)
    except Exception:
        return None


def committed_pipe_utilization(name: str):
    """Tensor-pipe (or FMA-pipe) utilisation of the dominant kernel for this configuration, from the committed
    ncu summary (profiles/pipe_utilization.json), if any."""
    p = os.path.join(ROOT, "profiles", "pipe_utilization.json")
    try:
        u = json.load(open(p)).get(name)
    except Exception:
        return None
    if isinstance(u, dict):
        u = dict(u, source="profiles/pipe_utilization.json: committed ncu capture of this configuration, "
                           "not measured in this run")
    return u


# ---- clock sampling during the timed region --------------------------------

class ClockSampler:
    """Samples the SM clock and the active clock-event reasons through NVML every ~20 ms."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int):
        self.samples: list[int] = []
        self.busy: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            self._sample_once()
            self._stop.wait(0.02)

    def _sample_once(self):
        nv = self._nv
        if nv is None:
            return
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
            self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.busy.append(nv.nvmlDeviceGetUtilizationRates(self._h).gpu)
        except Exception:
            pass

    def start(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._sample_once()
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        s = sorted(self.samples)
        b = self.busy
        names = [v for bit, v in self.REASONS.items() if self.reasons & bit and bit != 0x1]
        return {"sm_mhz": s[len(s) // 2], "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(s),
                "nvml_util_max_pct": max(b) if b else None}


# ---- distributed plumbing -----------------------------------------------------

def dist_setup(n_gpus: int):
    import torch

    if n_gpus <= 1 or "RANK" not in os.environ:
        torch.cuda.set_device(0)
        return 0, 1, 0, None
    import datetime

    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    # Bring the communicator up now and say how many ranks it spans (the log shows every rank's count).
    t = torch.ones(1, device="cuda")
    dist.all_reduce(t)
    torch.cuda.synchronize()
    print(f"[bench] rank {dist.get_rank()}: NCCL communicator up, nranks={int(t.item())} "
          f"(world_size {dist.get_world_size()}, NCCL {'.'.join(map(str, torch.cuda.nccl.version()))})",
          file=sys.stderr, flush=True)
    return dist.get_rank(), dist.get_world_size(), local, dist


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(dist, values: list) -> list:
    """Every rank's `values` (floats), in rank order; [values] without a process group."""
    if dist is None:
        return [list(values)]
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device="cuda")
    out = torch.empty(t.numel() * dist.get_world_size(), dtype=torch.float64, device="cuda")
    dist.all_gather_into_tensor(out, t)
    return out.view(dist.get_world_size(), -1).tolist()


def sum_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(dist):
    import torch

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ---- our implementation ----------------------------------------------------------

def rank_share(cfg: dict, rank: int, world: int, scaling: str):
    """This rank's share and its Shard: weak scaling keeps one configuration's worth of work per
    rank (the global problem grows with the world), strong scaling splits one configuration."""
    import sharding

    c = dict(cfg)
    if cfg["shard"] == "batch":
        total = cfg["batch"] * (world if scaling == "weak" else 1)
        s = sharding.plan(total, world, rank, "batch", 1)
        c["batch"] = s.size
    else:
        total = cfg["n"] * (world if scaling == "weak" else 1)
        s = sharding.plan(total, world, rank, "cols", 256)
        c["n"] = s.size
    return c, s


def make_inputs(cfg: dict, seed: int):
    """Seeded synthetic operands on the current device (configuration value distributions)."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    dt = cfg["dt"]
    na, nb, nc = m * k * b, k * n * b, m * n * b
    if dt == 3:
        A = torch.randint(-128, 128, (na,), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
        B = torch.randint(-128, 128, (nb,), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
        C = torch.zeros(nc, device="cuda", dtype=torch.int32)
    elif dt == 0:
        A = torch.rand(na, generator=g, device="cuda") * 2 - 1
        B = torch.rand(nb, generator=g, device="cuda") * 2 - 1
        C = torch.rand(nc, generator=g, device="cuda") * 2 - 1
    else:
        tdt = torch.float16 if dt == 2 else torch.bfloat16
        A = (torch.randn(na, generator=g, device="cuda") * 0.25).to(tdt)
        B = (torch.randn(nb, generator=g, device="cuda") * 0.25).to(tdt)
        C = torch.zeros(nc, device="cuda", dtype=torch.float32)
    return A, B, C


def call(h, cfg: dict, A, B, C):
    """One step through the cuBLAS-shaped device entry point."""
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    ta, tb = cfg["op"]
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    if cfg["api"] == "sgemm":
        h.sgemm(ta, tb, m, n, k, cfg["alpha"], A, lda, B, ldb, cfg["beta"], C, m)
    elif cfg["api"] == "strided":
        h.gemm_strided_batched_ex(ta, tb, m, n, k, cfg["alpha"], A, cfg["dt"], lda, m * k, B, cfg["dt"], ldb, k * n,
                                  cfg["beta"], C, cfg["ct"], m, m * n, b, cfg["comp"], algo=cfg.get("algo", -1))
    else:
        h.gemm_ex(ta, tb, m, n, k, cfg["alpha"], A, cfg["dt"], lda, B, cfg["dt"], ldb, cfg["beta"], C, cfg["ct"], m,
                  cfg["comp"], algo=cfg.get("algo", -1))


def call_host(h, cfg: dict, Ah, Bh, Ch):
    """One step through the host-buffer entry point (gs_host_gemm_ex): H2D, compute, D2H."""
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    ta, tb = cfg["op"]
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    h.host_gemm_ex(ta, tb, m, n, k, cfg["alpha"], Ah, cfg["dt"], lda, Bh, cfg["dt"], ldb, cfg["beta"], Ch, cfg["ct"],
                   m, cfg["comp"], batch=b)


def l2_flush_needed(cfg: dict) -> bool:
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    largest = max(m * k, k * n) * b * ELEM[cfg["dt"]]
    return largest <= 126 * 2 ** 20


def config_dict(cfg0: dict, cfg: dict, world: int, scaling: str, shard_of: int = 0) -> dict:
    """The `config` object of a result line; both arms print the same one for the same workload."""
    parts = world if world > 1 else shard_of
    d = {"workload": cfg0["label"], "name": cfg0["name"],
         "per_rank": {"m": cfg["m"], "n": cfg["n"], "k": cfg["k"], "batch": cfg["batch"]},
         "sharding": "none" if parts <= 1 else (f"{cfg0['shard']} split, {scaling} scaling, "
                                                "no data-path collective"),
         "l2": "flushed (256 MiB write) before every step" if l2_flush_needed(cfg)
         else "inputs larger than L2 (126 MB)"}
    if shard_of > 1 and world == 1:
        d["emulated_shard"] = f"rank 0's share of a {shard_of}-way {scaling} split, run alone on one GPU"
    return d


def run_ours(args, items: list) -> None:
    """Our arm: every (configuration, scaling) item in one process group, one JSON line per item."""
    import torch

    import gemm_sm100 as gs

    rank, world, local, dist = dist_setup(args.gpus)
    peaks = load_peaks()
    stream = torch.cuda.current_stream()
    h = gs.Handle(stream=stream)
    try:
        for cfg_name, scaling in items:
            line = run_ours_one(args, h, stream, peaks, rank, world, local, dist, cfg_name, scaling)
            if rank == 0:
                emit(line)
            torch.cuda.empty_cache()
    finally:
        h.close()
        if dist is not None:
            dist.destroy_process_group()


def run_ours_one(args, h, stream, peaks, rank, world, local, dist, cfg_name: str, scaling: str) -> dict:
    import torch

    cfg0 = dict(CONFIGS[cfg_name], algo=args.algo, name=cfg_name)
    parts = world if world > 1 else max(1, args.shard_of)
    cfg, shard = rank_share(cfg0, rank, parts, scaling)
    A, B, C = make_inputs(cfg, seed=1234 + rank)
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device="cuda") if l2_flush_needed(cfg) else None

    def step():
        if flush is not None:
            flush.zero_()
        call(h, cfg, A, B, C)

    for _ in range(args.warmup):
        step()
    barrier(dist)
    sampler = ClockSampler(local)
    launches0 = h.launch_count()
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host_t0 = time.perf_counter()
    if flush is None:
        ev0.record(stream)
        for _ in range(args.steps):
            call(h, cfg, A, B, C)
        ev1.record(stream)
        torch.cuda.synchronize()
        elapsed = ev0.elapsed_time(ev1)
        kernel_ms = elapsed / max(1, args.steps)
    else:
        # L2 is flushed between steps; the GEMM launch alone is timed per step.
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        ev0.record(stream)
        for s0, s1 in evs:
            flush.zero_()
            s0.record(stream)
            call(h, cfg, A, B, C)
            s1.record(stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        kernel_ms = sum(s0.elapsed_time(s1) for s0, s1 in evs) / max(1, args.steps)
        elapsed = kernel_ms * args.steps
    host_ms = (time.perf_counter() - host_t0) * 1e3
    # share of the timed region's host wall time (launches through the final synchronize) that this rank's
    # GPU spent in the timed kernels
    busy = min(1.0, elapsed / host_ms) if host_ms > 0 else 0.0
    clocks = sampler.stop()
    launches = h.launch_count() - launches0
    dev_err = h.device_error()
    barrier(dist)
    per_rank = all_ranks(dist, [kernel_ms, busy, clocks.get("sm_mhz") or -1.0])
    max_elapsed = max_over_ranks(dist, elapsed)
    max_kernel_ms = max_over_ranks(dist, kernel_ms)
    flops_rank, bytes_rank = work(cfg)
    total_flops = sum_over_ranks(dist, flops_rank)
    ms_per_step = max_elapsed / max(1, args.steps)
    value = total_flops / (ms_per_step * 1e-3) / 1e12

    # ---- end to end through the host-buffer entry point ----
    e2e_ms = e2e_value = None
    if not args.no_e2e:
        Ah = A.cpu().pin_memory()
        Bh = B.cpu().pin_memory()
        Ch = C.cpu().pin_memory()
        e2e_steps = max(1, min(args.steps, 20))
        call_host(h, cfg, Ah, Bh, Ch)  # warm the staging buffers
        barrier(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            call_host(h, cfg, Ah, Bh, Ch)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1)) / e2e_steps
        e2e_value = total_flops / (e2e_ms * 1e-3) / 1e12
        del Ah, Bh, Ch
    h2d = A.numel() * A.element_size() + B.numel() * B.element_size()
    if cfg["beta"] != 0:
        h2d += C.numel() * C.element_size()
    d2h = C.numel() * C.element_size()

    roof = roofline_of(cfg, flops_rank, bytes_rank, max_kernel_ms, peaks, committed_traffic(cfg_name))
    unit = "TOP/s" if cfg["dt"] == 3 else "TFLOP/s"
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": scaling if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": DTYPE_NAME[cfg["dt"]],
        "data": "synthetic (seeded torch generator; value distributions of the configuration)",
        "config": config_dict(cfg0, cfg, world, scaling, 0 if world > 1 else args.shard_of),
        "e2e": {"value": round(e2e_value, 2), "unit": unit, "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world, "ms_per_step": round(e2e_ms, 3),
                "path": "gs_host_gemm_ex (pinned host buffers; H2D, kernel, D2H, stream sync per step)"}
        if e2e_value is not None else {"skipped": "--no-e2e (a profiling run)"},
        "roofline": roof,
        "pipe_utilization": committed_pipe_utilization(cfg_name),
        "gpu_launches": int(launches),
        "device_busy": round(busy, 4),
        "clocks": clocks,
        "device_error_word": dev_err,
        "kernels": h.last_kernels(),
    }
    if world > 1:
        import torch.distributed as tdist

        line["ranks"] = {"kernel_ms": [round(r[0], 4) for r in per_rank],
                         "device_busy": [round(r[1], 4) for r in per_rank],
                         "sm_mhz": [r[2] if r[2] >= 0 else None for r in per_rank],
                         "units": [shard.cuts[g + 1] - shard.cuts[g] for g in range(world)],
                         "unit": "columns" if cfg0["shard"] == "cols" else "batch entries"}
        line["nccl"] = {"nranks": tdist.get_world_size(), "version": ".".join(map(str, torch.cuda.nccl.version()))}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg0, budget_s=args.cpu_seconds)
    if args.gather and dist is not None:
        # Optional NCCL all-gather of the C blocks onto every rank, timed on its own
        # (not part of `value`: the sharded GEMM itself needs no collective).
        import sharding

        unit_elems = cfg["m"] if cfg0["shard"] == "cols" else cfg["m"] * cfg["n"]
        sharding.gather_blocks(C, shard, unit_elems)  # warm the communicator
        barrier(dist)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        full = sharding.gather_blocks(C, shard, unit_elems)
        g1.record(stream)
        torch.cuda.synchronize()
        gms = max_over_ranks(dist, g0.elapsed_time(g1))
        nbytes = int(full.numel() * full.element_size())
        line["allgather"] = {"ms": round(gms, 3), "bytes_per_rank": nbytes, "backend": "nccl",
                             "algbw_gbs": round(nbytes * (world - 1) / world / (gms * 1e-3) / 1e9, 1)}
        del full
    if args.cublas:
        # Every rank runs cuBLAS on its own shard, so that all GPUs carry the same work (and heat) into the
        # next item; rank 0's result is reported.
        cub = cublas_compare(cfg, A, B, args.steps, args.warmup, flush)
        if rank == 0:
            line["cublas"] = cub
            if "ms" in cub:
                # the reference's shader_cublas_ratio (bench/gemm_perf.zig:206): our ms / cuBLAS ms, rank-0 shard
                line["shader_cublas_ratio"] = round(max_kernel_ms / cub["ms"], 4)
    del A, B, C, flush
    return line


def cublas_compare(cfg: dict, A, B, steps: int, warmup: int, flush=None) -> dict:
    """cuBLAS on the same operands and arguments (cublasGemmEx / cublasGemmStridedBatchedEx, as
    slang-gemm's src/cublas.zig calls them), timed like our kernel, for shader_cublas_ratio: back to back
    when the operands are larger than L2, else with `flush` (the same 256 MiB buffer) written before every
    call and each call timed on its own."""
    import torch

    import cublas_ref

    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    ta, tb = cfg["op"]
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    C2 = torch.zeros(m * n * b, device="cuda", dtype=torch.int32 if cfg["ct"] == 10 else torch.float32)
    stream = torch.cuda.current_stream()
    cb = cublas_ref.Cublas(stream=stream)
    fn = lambda: cb.gemm_strided_batched_ex(ta, tb, m, n, k, cfg["alpha"], A, cfg["dt"], lda, m * k, B, cfg["dt"],  # noqa
                                            ldb, k * n, cfg["beta"], C2, cfg["ct"], m, m * n, b, cfg["comp"])
    status = fn()
    if status != 0:
        return {"note": f"cublasGemmEx returned {status}", "version": cublas_ref.version_string()}
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for s0, s1 in evs:
            flush.zero_()
            s0.record(stream)
            fn()
            s1.record(stream)
        torch.cuda.synchronize()
        ms = sum(s0.elapsed_time(s1) for s0, s1 in evs) / max(1, steps)
    cb.close()
    unit = "TOP/s" if cfg["dt"] == 3 else "TFLOP/s"
    return {"ms": round(ms, 4), "value": round(2.0 * m * n * k * b / ms / 1e9, 1), "unit": unit,
            "l2": "inputs larger than L2" if flush is None else "flushed before every call, as ours",
            "call": "cublasGemmStridedBatchedEx" if b > 1 else "cublasGemmEx",
            "version": cublas_ref.version_string()}


def run_sustained(args, cfg_name: str) -> None:
    """Power-capped steady state: libgemm_sm100 and cuBLAS each run back-to-back calls for `--sustained`
    seconds (alternating, twice), with NVML clock / power / throttle-reason samples every 10 ms. Prints one
    JSON line (mode "sustained"), not the contract line: it shows the clock each library settles at under the
    1 kW cap, which a 50-step burst does not reach."""
    import torch

    import cublas_ref
    import gemm_sm100 as gs

    cfg = dict(CONFIGS[cfg_name], algo=args.algo)
    torch.cuda.set_device(0)
    A, B, C = make_inputs(cfg, seed=1)
    stream = torch.cuda.current_stream()
    h = gs.Handle(stream)
    cb = cublas_ref.Cublas(stream=stream)
    m, n, k, b = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    ta, tb = cfg["op"]
    lda, ldb = (m if ta == 0 else k), (k if tb == 0 else n)
    C2 = torch.zeros_like(C)
    theirs = lambda: cb.gemm_strided_batched_ex(ta, tb, m, n, k, cfg["alpha"], A, cfg["dt"], lda, m * k, B,  # noqa
                                                cfg["dt"], ldb, k * n, cfg["beta"], C2, cfg["ct"], m, m * n, b,
                                                cfg["comp"])
    ours = lambda: call(h, cfg, A, B, C)  # noqa: E731
    flops = 2.0 * m * n * k * b
    try:
        import pynvml

        pynvml.nvmlInit()
        nvh = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
    except Exception:
        pynvml = None
    rows = []
    for rep in range(2):
        for name, fn in (("libgemm_sm100", ours), ("cuBLAS", theirs)):
            fn()
            torch.cuda.synchronize()
            t0 = time.time()
            fn()
            torch.cuda.synchronize()
            iters = max(5, int(args.sustained / max(time.time() - t0, 1e-4)))
            samples, stop = [], threading.Event()

            def sample():
                while pynvml is not None and not stop.is_set():
                    try:
                        samples.append((pynvml.nvmlDeviceGetClockInfo(nvh, pynvml.NVML_CLOCK_SM),
                                        pynvml.nvmlDeviceGetPowerUsage(nvh) / 1000.0,
                                        pynvml.nvmlDeviceGetCurrentClocksEventReasons(nvh)))
                    except Exception:
                        pass
                    stop.wait(0.01)

            th = threading.Thread(target=sample, daemon=True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            th.start()
            e0.record(stream)
            for _ in range(iters):
                fn()
            e1.record(stream)
            e1.synchronize()
            stop.set()
            th.join()
            ms = e0.elapsed_time(e1) / iters
            mid = samples[len(samples) // 4: 3 * len(samples) // 4] or samples
            reasons = 0
            for s in mid:
                reasons |= s[2]
            med = lambda xs: sorted(xs)[len(xs) // 2] if xs else None  # noqa: E731
            rows.append({"impl": name, "rep": rep, "calls": iters, "ms": round(ms, 4),
                         "value": round(flops / ms / 1e9, 1), "sm_mhz_median": med([s[0] for s in mid]),
                         "power_w_median": None if not mid else round(med([s[1] for s in mid]), 1),
                         "reasons": [v for bit, v in ClockSampler.REASONS.items() if reasons & bit]})
            time.sleep(1.0)
    cb.close()
    emit({"mode": "sustained", "config": {"name": cfg_name, "workload": cfg["label"]}, "seconds": args.sustained,
          "unit": "TOP/s" if cfg["dt"] == 3 else "TFLOP/s", "cublas_version": cublas_ref.version_string(),
          "rows": rows})


# ---- CPU legs: the reference's scalar algorithm (oracle port) ----------------------

def _oracle():
    sys.path.insert(0, ORACLE_DIR)
    import oracle

    return oracle


def _cpu_sample(cfg: dict, cols: int, threads: int, seed: int = 7) -> float:
    """Seconds for the oracle to compute `cols` full columns of C (all M rows, full K)."""
    import numpy as np

    orc = _oracle()
    rng = np.random.default_rng(seed)
    m, k = cfg["m"], cfg["k"]
    ta, tb = cfg["op"]
    dt, ct = cfg["dt"], cfg["ct"]
    if not hasattr(_cpu_sample, "cache") or _cpu_sample.cache[0] != (m, k, dt):
        if dt == 3:
            a = rng.integers(-128, 128, m * k).astype(np.int8)
        elif dt == 0:
            a = rng.uniform(-1, 1, m * k).astype(np.float32)
        else:
            a = orc.randn_lowp(rng, m * k, dt)
        _cpu_sample.cache = ((m, k, dt), a)
    a = _cpu_sample.cache[1]
    if dt == 3:
        b = rng.integers(-128, 128, k * cols).astype(np.int8)
        c = np.zeros(m * cols, np.int32)
    elif dt == 0:
        b = rng.uniform(-1, 1, k * cols).astype(np.float32)
        c = rng.uniform(-1, 1, m * cols).astype(np.float32)
    else:
        b = orc.randn_lowp(rng, k * cols, dt)
        c = np.zeros(m * cols, np.float32)
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else cols
    t0 = time.perf_counter()
    if cfg["api"] == "sgemm":
        rc = orc.sgemm_strided_batched_mt(orc.COL_MAJOR, ta, tb, m, cols, k, cfg["alpha"], a, lda, 0, b, ldb, 0,
                                          cfg["beta"], c, m, 0, 1, threads)
    else:
        rc = orc.gemm_ex(ta, tb, m, cols, k, cfg["alpha"], a, dt, lda, b, dt, ldb, cfg["beta"], c, ct, m,
                         compute_type=cfg["comp"], threads=threads)
    dt_s = time.perf_counter() - t0
    assert rc == orc.OK
    return dt_s


def _cpu_plan(cfg: dict, threads: int, budget_s: float) -> tuple[int, float]:
    """Columns per sample so that one sample takes about budget_s seconds."""
    t1 = _cpu_sample(cfg, threads, threads)
    per = max(1, int(budget_s / max(t1, 1e-6)))
    return threads * per, t1


def cpu_single_thread(cfg: dict) -> dict:
    """Single-thread scalar figures of the oracle's loop: (i) the whole GEMM at the reference bench's capped
    size (min(dim, 256) for classic sgemm, min(dim, 128) for gemmEx; bench/gemm_perf.zig:317-336, :618-637),
    as the reference times its scalar column; (ii) the full-size GEMM when it is small enough (C1's 512^3),
    otherwise a two-column sample of it."""
    cap = 256 if cfg["api"] == "sgemm" else 128
    small = dict(cfg, m=min(cfg["m"], cap), n=min(cfg["n"], cap), k=min(cfg["k"], cap), batch=1)
    secs_cap = _cpu_sample(small, small["n"], 1)
    full = cfg["m"] * cfg["n"] * cfg["k"] <= 2 ** 28
    cols = cfg["n"] if full else 2
    secs = _cpu_sample(cfg, cols, 1)
    unit = "TOP/s" if cfg["dt"] == 3 else "TFLOP/s"
    f_cap = 2.0 * small["m"] * small["n"] * small["k"]
    f_full = 2.0 * cfg["m"] * cols * cfg["k"]
    return {"value": f_full / secs / 1e12, "unit": unit, "cores": 1,
            "sample": (f"the whole {cfg['m']}x{cfg['n']}x{cfg['k']} GEMM" if full else
                       f"{cols} of {cfg['n']} output columns of the {cfg['m']}x{cfg['n']}x{cfg['k']} GEMM")
            + f", {secs:.2f} s",
            "ms_full_gemm_estimate": round(secs * 1e3 * cfg["n"] / cols * cfg["batch"], 1),
            "at_reference_cap": {"m": small["m"], "n": small["n"], "k": small["k"], "ms": round(secs_cap * 1e3, 3),
                                 "value": f_cap / secs_cap / 1e12, "unit": unit}}


def cpu_baseline(cfg: dict, budget_s: float = 12.0) -> dict:
    """The C restatement of the reference's scalar gemmExCuda (src/gemm.zig:671-706), all host cores, plus the
    single-thread scalar figures beside it."""
    threads = os.cpu_count() or 1
    cols, _ = _cpu_plan(cfg, threads, budget_s)
    cols = min(cols, cfg["n"])
    secs = _cpu_sample(cfg, cols, threads)
    flops = 2.0 * cfg["m"] * cols * cfg["k"]
    unit = "TOP/s" if cfg["dt"] == 3 else "TFLOP/s"
    return {"value": flops / secs / 1e12, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{cols} of {cfg['n']} output columns (all {cfg['m']} rows, full K={cfg['k']}) of one "
                      f"{cfg['m']}x{cfg['n']}x{cfg['k']} GEMM, {secs:.1f} s, {threads} threads "
                      "(oracle/gemm_oracle.c, the scalar f64-accumulating loop of src/gemm.zig)",
            "single_thread": cpu_single_thread(cfg)}


def rank0_units(units: int, parts: int, align: int) -> int:
    """Rank 0's share under gs_plan_shards's cut rule (floor(units * g / parts) rounded down to `align`)."""
    if parts <= 1:
        return units
    return (units // parts) // align * align


def run_reference(args, cfg_name: str, scaling: str = "weak") -> None:
    """--impl reference: the reference's CPU algorithm on this host, same config / metric / unit."""
    if int(os.environ.get("RANK", "0")) != 0:
        return  # only rank 0 runs and prints under torchrun
    cfg = dict(CONFIGS[cfg_name], name=cfg_name)
    world = int(os.environ.get("WORLD_SIZE", "1")) if "RANK" in os.environ else 1
    threads = os.cpu_count() or 1
    total_steps = args.steps + args.warmup
    per_step_budget = max(0.5, args.ref_seconds / max(1, total_steps))
    cols, _ = _cpu_plan(cfg, threads, per_step_budget)
    cols = min(cols, cfg["n"])
    for _ in range(args.warmup):
        _cpu_sample(cfg, cols, threads)
    t = 0.0
    for _ in range(args.steps):
        t += _cpu_sample(cfg, cols, threads)
    flops = 2.0 * cfg["m"] * cols * cfg["k"] * args.steps
    value = flops / t / 1e12
    unit = "TOP/s" if cfg["dt"] == 3 else "TFLOP/s"
    frac = cols / cfg["n"]
    sample = (f"{cols} of {cfg['n']} output columns per step (all {cfg['m']} rows, full K={cfg['k']}), "
              f"{threads} threads, oracle/gemm_oracle.c (C restatement of src/gemm.zig gemmExCuda; "
              "the Zig reference itself cannot be built here)")
    # Same `config` object as our arm prints for this workload (rank 0's share when N > 1), computed here
    # without loading libgemm_sm100: this arm runs none of this repository's GPU code.
    rcfg = dict(cfg)
    if world > 1:
        key, align = ("batch", 1) if cfg["shard"] == "batch" else ("n", 256)
        total = cfg[key] * (world if scaling == "weak" else 1)
        rcfg[key] = rank0_units(total, world, align)
    # ms_per_step describes the same work as `value`: one whole step of the configuration (per batch entry
    # count and full N), extrapolated from the timed column sample at the sampled rate.
    ms_full = 1000.0 * t / max(1, args.steps) / frac * cfg["batch"]
    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_full, 1), "higher_is_better": True,
        "scaling": scaling if world > 1 else "weak", "vs_baseline": None, "dtype": DTYPE_NAME[cfg["dt"]],
        "data": "synthetic (seeded numpy generator; value distributions of the configuration)",
        "config": config_dict(cfg, rcfg, world, scaling),
        "impl": "reference",
        "sample_fraction": round(frac * (1.0 / cfg["batch"]), 6),
        "ms_per_sample": round(1000.0 * t / max(1, args.steps), 1),
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# The result line is the only thing written to stdout: libraries that print
# banners (NCCL, for one) see stderr as their stdout while bench.py runs.
_RESULT_FD = None


def emit(line: dict) -> None:
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, data)


# ---- manifest rows (the reference's JSONL harness, bench/gemm_perf.zig) ----------------

def _manifest_scalar_fn(case):
    """CPU scalar column of a manifest row: the oracle (single thread) at the reference bench's capped sizes,
    256 for classic sgemm and 128 for Ex rows, 2 batch entries for batched Ex rows
    (bench/gemm_perf.zig:317-336, :618-637, :729-774)."""
    import numpy as np

    import manifest as mf
    import perf_rows as pr

    orc = _oracle()
    s = case.shape
    cap = 256 if case.api in mf.CLASSIC_APIS else 128
    m, n, k = min(s.m, cap), min(s.n, cap), min(s.k, cap)
    batch = 2 if case.api in ("gemm_batched_ex", "gemm_strided_batched_ex") else 1
    ar, ac = pr.stored_dims(case.op_a, m, k)
    br, bc = pr.stored_dims(case.op_b, k, n)
    opa, opb = mf.OP_VALUE[case.op_a], mf.OP_VALUE[case.op_b]
    at, bt, ct, comp = case.type_codes()
    if case.api in mf.CLASSIC_APIS:
        a, b, c = pr.fill_f32(ar * ac, 0.1), pr.fill_f32(br * bc, -0.2), pr.fill_f32(m * n, 0.3)
        t0 = time.perf_counter()
        rc = orc.sgemm(orc.COL_MAJOR, opa, opb, m, n, k, 1.0, a, ar, b, br, 0.0, c, m)
        ms = (time.perf_counter() - t0) * 1e3
    else:
        sa, sb, sc = ar * ac, br * bc, m * n
        if case.a_type == mf.R8I:
            a, b = pr.fill_i8(sa * batch, 1), pr.fill_i8(sb * batch, -2)
        elif case.a_type in (mf.R16F, mf.R16BF):
            a, b = pr.fill_lowp16(sa * batch, case.a_type, 0.1), pr.fill_lowp16(sb * batch, case.a_type, -0.2)
        else:
            a, b = pr.fill_f32(sa * batch, 0.1), pr.fill_f32(sb * batch, -0.2)
        c = {mf.R32I: np.zeros(sc * batch, np.int32), mf.R16F: np.zeros(sc * batch, np.uint16)}.get(
            case.c_type, np.zeros(sc * batch, np.float32))
        t0 = time.perf_counter()
        rc = orc.gemm_ex(opa, opb, m, n, k, 1.0, a, at, ar, b, bt, br, 0.0, c, ct, m, compute_type=comp,
                         layout=orc.COL_MAJOR, batch=batch, sa=sa, sb=sb, sc=sc)
        ms = (time.perf_counter() - t0) * 1e3
    if rc != 0:
        return None
    return ms, (m, n, k, batch)


def run_manifest(args):
    """JSONL rows + summary line of the reference's benchmark CLI (bench/gemm_perf.zig:50-89), for this backend:
    shader_* columns are libgemm_sm100, cublas_* the vendor library on the same buffers, scalar_* the oracle."""
    import torch

    import manifest as mf
    import perf_rows as pr

    if not torch.cuda.is_available():
        emit({"status": "invalid", "error": "no CUDA device available"})
        return 0
    if args.device_substr:
        names = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
        idx = next((i for i, nm in enumerate(names) if args.device_substr in nm), None)
        if idx is None:
            emit({"status": "invalid", "error": f"no CUDA device name contains {args.device_substr!r}"})
            return 1
        torch.cuda.set_device(idx)
    sizes = [int(x) for x in args.sizes.split(",") if x.strip()] if args.sizes else [512, 1024, 2048]
    rects = []
    for item in (args.rect_sizes or "").split(","):
        if item.strip():
            m, n, k = (int(v) for v in item.lower().split("x"))
            rects.append(mf.Shape(m, n, k))
    out = open(args.output, "w") if args.output else None

    def write(row):
        line = json.dumps(row)
        if out:
            out.write(line + "\n")
            out.flush()
        else:
            emit(row)

    runner = pr.Runner(write, warmup=args.warmup, iters=args.iters, fail_every_row=args.fail_every_row,
                       only_cublas_supported=args.only_cublas_supported,
                       tile_compatible_only=args.tile_compatible_only,
                       scalar_fn=None if args.no_cpu_baseline else _manifest_scalar_fn)
    summary = runner.run(sizes, rects, args.manifest == "all")
    if out:
        out.close()
    geo = summary.geomean()
    if args.fail_on_regression and geo is not None and geo > 1.0:
        return 1
    if args.fail_every_row and summary.strict_failures:
        return 1
    return 0


# Shapes of the tile-choice sweep (M, N, K, batch) and of the split-K comparison.
TILE_SWEEP_SHAPES = [
    (8192, 8192, 8192, 1), (4096, 4096, 4096, 1), (2048, 2048, 2048, 1), (8192, 8192, 1024, 1), (4096, 4096, 1024, 1),
    (8192, 1024, 8192, 1), (1024, 8192, 8192, 1), (3000, 3000, 3000, 1), (6144, 6144, 2048, 1), (2048, 8192, 4096, 1),
    (8192, 2048, 512, 1), (1536, 1536, 1536, 1), (512, 512, 16384, 1), (16384, 4096, 1024, 1), (1024, 1024, 1024, 1),
    (512, 512, 1024, 256), (2048, 2048, 2048, 64), (1024, 1024, 1024, 32), (256, 256, 4096, 128), (768, 768, 768, 64),
    (4096, 4096, 256, 8), (2048, 2048, 1536, 16), (2560, 2560, 2560, 1), (3072, 3072, 1024, 1), (1024, 4096, 2048, 1),
    (4096, 2048, 2048, 1), (1024, 1024, 4096, 1), (2048, 2048, 512, 1), (512, 512, 512, 64), (1024, 1024, 256, 64),
    (2048, 1024, 1024, 16), (384, 384, 1024, 128), (1280, 1280, 1280, 8), (8192, 4096, 256, 1), (512, 512, 768, 64),
    (512, 1024, 512, 96)]
SPLITK_SHAPES = [(512, 512, 16384, 1), (1024, 1024, 4096, 1), (1024, 1024, 8192, 1), (256, 1024, 32768, 1),
                 (2048, 512, 8192, 1), (768, 768, 12288, 1)]


def run_tile_sweep(args) -> int:
    """Every tensor-core tile against the automatic choice, and cuBLAS, over a list of shapes (op N/N, alpha 1,
    beta 0). The five calls of a shape (algo -1 automatic, 0 = 1-SM 128x256, 1 = pair 256x256, 2 = wide 256x512,
    cuBLAS) are timed in turn, 7 times, each time as a run of back-to-back calls of about 2 ms after a 256 MiB L2
    flush (the event clock ticks in ~2 us steps here, so short calls are not timed one by one); the medians of
    the per-call times are printed, one JSON line per shape, with whether the automatic call split K."""
    import torch

    import cublas_ref
    import gemm_sm100 as gs

    torch.cuda.set_device(0)
    h = gs.Handle()
    cb = cublas_ref.Cublas(stream=torch.cuda.current_stream())
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device="cuda")

    def run_of(fn, r):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(r):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / r

    shapes = SPLITK_SHAPES if args.tile_sweep == "splitk" else TILE_SWEEP_SHAPES
    if args.sweep_shapes:
        shapes = [tuple(int(v) for v in x.split("x")) + ((1,) if x.count("x") == 2 else ()) for x in
                  args.sweep_shapes.split(",")]
    types = {"f16": (gs.R_16F, gs.R_32F, gs.COMPUTE_32F), "bf16": (gs.R_16BF, gs.R_16BF, gs.COMPUTE_32F),
             "i8": (gs.R_8I, gs.R_32I, gs.COMPUTE_32I)}
    for dname in args.sweep_dtypes.split(","):
        at, ct, comp = types[dname]
        for m, n, k, b in shapes:
            if at == gs.R_8I and (m % 16 or k % 16):
                continue  # not TMA-addressable: the CUDA-core path, no tile to compare
            g = torch.Generator(device="cuda").manual_seed(m + n + k + b)
            if at == gs.R_8I:
                A = torch.randint(-128, 128, (b * m * k,), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
                B = torch.randint(-128, 128, (b * k * n,), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
                C = torch.zeros(b * m * n, dtype=torch.int32, device="cuda")
            else:
                tdt = torch.float16 if at == gs.R_16F else torch.bfloat16
                A = torch.randn(b * m * k, generator=g, device="cuda").to(tdt)
                B = torch.randn(b * k * n, generator=g, device="cuda").to(tdt)
                C = torch.zeros(b * m * n, dtype=torch.float32 if ct == gs.R_32F else tdt, device="cuda")
            C2 = C.clone()

            def ours(algo):
                return lambda: h.gemm_strided_batched_ex(0, 0, m, n, k, 1, A, at, m, m * k, B, at, k, k * n, 0, C, ct,
                                                         m, m * n, b, comp, algo=algo)

            fns = [ours(-1), ours(0), ours(1), ours(2),
                   lambda: cb.gemm_strided_batched_ex(0, 0, m, n, k, 1, A, at, m, m * k, B, at, k, k * n, 0, C2, ct,
                                                      m, m * n, b, comp)]
            for f in fns:
                f()
                f()
            torch.cuda.synchronize()
            r = max(3, min(200, int(2.0 / max(run_of(fns[0], 3), 1e-3))))
            ts = [[] for _ in fns]
            for _ in range(7):
                for i, f in enumerate(fns):
                    ts[i].append(run_of(f, r))
            med = [sorted(x)[3] for x in ts]
            fns[0]()
            kern = h.last_kernels()
            st, tile, parts = gs.plan_tile(0, 0, m, n, k, at, ct, comp, batch=b)
            best = min(med[1:4])
            emit({"mode": "tile-sweep", "dt": dname, "m": m, "n": n, "k": k, "batch": b,
                  "auto_ms": round(med[0], 5), "tile_1sm_ms": round(med[1], 5), "tile_pair_ms": round(med[2], 5),
                  "tile_wide_ms": round(med[3], 5), "cublas_ms": round(med[4], 5),
                  "auto_tile": tile, "auto_k_slices": parts, "split_k": bool(kern & gs.KERNEL_REDUCE),
                  "best_tile": 1 + min(range(3), key=lambda i: med[1 + i]), "auto_over_best": round(med[0] / best, 4),
                  "auto_over_cublas": round(med[0] / med[4], 4)})
            del A, B, C, C2
            torch.cuda.empty_cache()
    return 0


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3-f16-nn",
                    help="configuration name, or a comma-separated list (one JSON line each): "
                         + ", ".join(sorted(CONFIGS)))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="weak",
                    help="N > 1: 'weak' (each rank holds one configuration's work), 'strong' (the ranks split one "
                         "configuration), or 'weak,strong' (both, one line each)")
    ap.add_argument("--shard-of", type=int, default=0, metavar="N",
                    help="one GPU runs rank 0's share of an N-way split alone (the per-rank workload of an N-GPU "
                         "run, for single-GPU profiling)")
    ap.add_argument("--no-cublas", dest="cublas", action="store_false",
                    help="skip timing cuBLAS on the same operands (shader_cublas_ratio)")
    ap.add_argument("--cublas", dest="cublas", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--gather", action="store_true", help="N > 1: also time an NCCL all-gather of C (separately)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling runs only)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target length of the cpu_baseline sample")
    ap.add_argument("--ref-seconds", type=float, default=90.0, help="target total length of --impl reference")
    ap.add_argument("--algo", type=int, default=-1,
                    help="cublasGemmAlgo_t passed to every call (a tile hint: 0 = 128x256, 1 = 256x256 pair, "
                         "2 = 256x512 pair; -1 = automatic)")
    ap.add_argument("--sustained", type=float, default=0.0, metavar="SECONDS",
                    help="instead of the contract line: power-capped steady state of this library vs cuBLAS")
    ap.add_argument("--tile-sweep", default=None, choices=["tiles", "splitk"],
                    help="instead of the contract line: every tensor-core tile against the automatic choice and "
                         "cuBLAS over the sweep's shapes ('tiles') or the split-K shapes ('splitk')")
    ap.add_argument("--sweep-shapes", default=None, help="--tile-sweep shapes, MxNxK[xBATCH] comma-separated")
    ap.add_argument("--sweep-dtypes", default="f16,i8", help="--tile-sweep input types: f16, bf16, i8")
    rows = ap.add_argument_group("manifest rows (the reference's JSONL benchmark CLI; any of these selects it)")
    rows.add_argument("--manifest", default=None, help="'all': every API/op/type case (bench/gemm_perf.zig:91)")
    rows.add_argument("--sizes", default=None, help="comma-separated square sizes (default 512,1024,2048)")
    rows.add_argument("--rect-sizes", default=None, help="comma-separated MxNxK shapes")
    rows.add_argument("--iters", type=int, default=20, help="timed calls per row")
    rows.add_argument("--fail-on-regression", action="store_true")
    rows.add_argument("--fail-every-row", action="store_true")
    rows.add_argument("--only-cublas-supported", action="store_true")
    rows.add_argument("--tile-compatible-only", action="store_true")
    rows.add_argument("--output", default=None, help="write rows to this file instead of stdout")
    rows.add_argument("--device-substr", default=None, help="first CUDA device whose name contains this")
    for accepted in ("--suite", "--ops", "--types"):
        rows.add_argument(accepted, default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    names = [c.strip() for c in args.config.split(",") if c.strip()]
    scalings = [s.strip() for s in args.scaling.split(",") if s.strip()]
    bad = [c for c in names if c not in CONFIGS] + [s for s in scalings if s not in ("weak", "strong")]
    if bad or not names or not scalings:
        ap.error(f"unknown --config / --scaling value(s): {bad}")
    args.config = names[0]
    row_mode = any(v is not None for v in (args.manifest, args.sizes, args.rect_sizes)) or args.fail_every_row or \
        args.fail_on_regression or args.only_cublas_supported or args.tile_compatible_only
    if row_mode:
        sys.exit(run_manifest(args))
    if args.tile_sweep:
        sys.exit(run_tile_sweep(args))
    if args.sustained:
        run_sustained(args, args.config)
        return
    if args.impl == "reference":
        run_reference(args, args.config, scalings[0])
    else:
        run_ours(args, [(c, s) for c in names for s in scalings])


if __name__ == "__main__":
    main()
