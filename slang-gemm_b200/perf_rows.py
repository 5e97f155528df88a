"""Manifest benchmark rows for the CUDA backend: one JSONL row per case with
cuBLAS and libgemm_sm100 timed on the same device buffers, plus the
reference's summary line.

Restates slang-gemm's bench/gemm_perf.zig row loop for this backend:
  - runCase / emitStatusOnly and the row schema: bench/gemm_perf.zig:192-244;
  - the summary line and the --fail-on-regression / --fail-every-row gates:
    bench/gemm_perf.zig:73-88;
  - the per-case timing (warm-up, then `iters` calls between two CUDA events,
    ms per call) and tflops = 2*m*n*k*batch / ms / 1e9:
    bench/gemm_perf.zig:300-316, :610-616, :1279-1282;
  - deterministic inputs: fill / fillLowp16 / fillI8 with the reference's
    biases (bench/gemm_perf.zig:1184-1189, :1227-1249), including that
    bench's own f32 -> f16 / bf16 conversion (round-half-up f16, truncated bf16).
"shader_ms" is this backend's kernel time per call. Unlike the Vulkan runner
(which never reads C back), every timed row also checks the result against
cuBLAS's on the same inputs (bit-exact for INT8, normwise relative error
otherwise) and reports status "validation_failed" when it disagrees.
The CPU scalar column is filled by a caller-supplied timer (`scalar_fn`); this
module never runs a CPU GEMM itself.
"""
from __future__ import annotations

import math

import numpy as np
import torch

import cublas_ref
import gemm_sm100 as gs
import manifest as mf

# Normwise tolerances against cuBLAS per output type (f32 from FP32 inputs, f16 output, bf16 inputs).
VALIDATION_TOL = {"f32": 1e-5, "f16_out": 2e-3, "lowp": 1e-2}


# ---- deterministic inputs (bench/gemm_perf.zig:1184-1249) -------------------------------------------------------
def fill_f32(count: int, bias: float) -> np.ndarray:
    i = np.arange(count, dtype=np.int64)
    return (((i * 19 + 7) % 23).astype(np.float32) - 11) / 7 + np.float32(bias)


def _f16_bits_round_half_up(v: np.ndarray) -> np.ndarray:
    """The reference bench's f32 -> f16 conversion (bench/gemm_perf.zig:1251-1262): adds half an ulp to the
    mantissa and truncates; subnormals by shifting the implicit-one mantissa."""
    bits = v.astype(np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xff) - 127 + 15
    man = bits & 0x7fffff
    out = sign | (np.clip(exp, 0, 31) << 10) | ((man + 0x1000) >> 13)
    sub = exp <= 0
    shift = np.clip(1 - exp, 0, 63)
    sub_val = sign | ((((man | 0x800000) >> shift) + 0x1000) >> 13)
    out = np.where(sub, np.where(exp < -10, sign, sub_val), out)
    out = np.where(exp >= 31, sign | 0x7c00, out)
    return out.astype(np.uint16)


def fill_lowp16(count: int, dtype: str, bias: float) -> np.ndarray:
    v = fill_f32(count, bias)
    if dtype == mf.R16F:
        return _f16_bits_round_half_up(v)
    return (v.view(np.uint32) >> 16).astype(np.uint16)  # bf16 by truncation, as that bench does


def fill_i8(count: int, bias: int) -> np.ndarray:
    i = np.arange(count, dtype=np.int64)
    return (((i * 7 + 3) % 17) - 8 + bias).astype(np.int8)


def stored_dims(op: str, rows: int, cols: int) -> tuple[int, int]:
    """storedRows / storedCols (bench/gemm_perf.zig:1264-1276)."""
    return (rows, cols) if op == "N" else (cols, rows)


def tflops(m: int, n: int, k: int, ms: float, batch: int = 1) -> float:
    return 2.0 * m * n * k * batch / (ms * 1e9) if ms > 0 else 0.0


# ---- one case ---------------------------------------------------------------------------------------------------
class _Buffers:
    """Device operands of one case, built from the reference's fills."""

    def __init__(self, case: mf.Case, device):
        s, batch = case.shape, case.batch_count()
        self.ar, self.ac = stored_dims(case.op_a, s.m, s.k)
        self.br, self.bc = stored_dims(case.op_b, s.k, s.n)
        self.sa, self.sb, self.sc = self.ar * self.ac, self.br * self.bc, s.m * s.n
        na, nb, nc = self.sa * batch, self.sb * batch, self.sc * batch
        a_t = case.a_type
        if a_t == mf.R8I:
            A, B = fill_i8(na, 1), fill_i8(nb, -2)
        elif a_t in (mf.R16F, mf.R16BF):
            A, B = fill_lowp16(na, a_t, 0.1).view(np.int16), fill_lowp16(nb, a_t, -0.2).view(np.int16)
        else:
            A, B = fill_f32(na, 0.1), fill_f32(nb, -0.2)
        if case.c_type == mf.R32I:
            C = np.zeros(nc, np.int32)
        elif case.c_type == mf.R16F:
            C = _f16_bits_round_half_up(fill_f32(nc, 0.3)).view(np.int16)
        else:
            C = fill_f32(nc, 0.3)
        self.A = torch.from_numpy(np.ascontiguousarray(A)).to(device)
        self.B = torch.from_numpy(np.ascontiguousarray(B)).to(device)
        self.C0 = torch.from_numpy(np.ascontiguousarray(C)).to(device)
        self.C_ours = self.C0.clone()
        self.C_ref = self.C0.clone()
        self.batch = batch
        es = lambda t: t.element_size()  # noqa: E731
        if case.api == "gemm_batched_ex":
            def arr(t, stride):
                return torch.tensor([t.data_ptr() + i * stride * es(t) for i in range(batch)], dtype=torch.int64,
                                    device=device)
            self.Aarr, self.Barr = arr(self.A, self.sa), arr(self.B, self.sb)
            self.Carr_ours, self.Carr_ref = arr(self.C_ours, self.sc), arr(self.C_ref, self.sc)


def _alpha_beta(case: mf.Case):
    return 1, 0  # the reference bench times alpha = 1, beta = 0 for every row


def _calls(case: mf.Case, h: gs.Handle, cb: cublas_ref.Cublas, buf: _Buffers):
    """(ours, theirs): zero-argument callables issuing one call of the case's API on each library."""
    s = case.shape
    m, n, k = s.m, s.n, s.k
    ta, tb = mf.OP_VALUE[case.op_a], mf.OP_VALUE[case.op_b]
    alpha, beta = _alpha_beta(case)
    at, bt, ct, comp = case.type_codes()
    lda, ldb, ldc = buf.ar, buf.br, m
    batch = buf.batch
    if case.api in mf.CLASSIC_APIS:
        if batch == 1:
            ours = lambda: h.sgemm(ta, tb, m, n, k, alpha, buf.A, lda, buf.B, ldb, beta, buf.C_ours, ldc)  # noqa
        else:
            ours = lambda: h.sgemm_strided_batched(ta, tb, m, n, k, alpha, buf.A, lda, buf.sa, buf.B, ldb,  # noqa
                                                   buf.sb, beta, buf.C_ours, ldc, buf.sc, batch)
        theirs = lambda: cb.sgemm(ta, tb, m, n, k, alpha, buf.A, lda, buf.B, ldb, beta, buf.C_ref, ldc,  # noqa
                                  buf.sa, buf.sb, buf.sc, batch)
    elif case.api == "gemm_ex":
        ours = lambda: h.gemm_ex(ta, tb, m, n, k, alpha, buf.A, at, lda, buf.B, bt, ldb, beta, buf.C_ours, ct,  # noqa
                                 ldc, comp)
        theirs = lambda: cb.gemm_strided_batched_ex(ta, tb, m, n, k, alpha, buf.A, at, lda, 0, buf.B, bt, ldb,  # noqa
                                                    0, beta, buf.C_ref, ct, ldc, 0, 1, comp)
    elif case.api == "gemm_strided_batched_ex":
        ours = lambda: h.gemm_strided_batched_ex(ta, tb, m, n, k, alpha, buf.A, at, lda, buf.sa, buf.B, bt,  # noqa
                                                 ldb, buf.sb, beta, buf.C_ours, ct, ldc, buf.sc, batch, comp)
        theirs = lambda: cb.gemm_strided_batched_ex(ta, tb, m, n, k, alpha, buf.A, at, lda, buf.sa, buf.B, bt,  # noqa
                                                    ldb, buf.sb, beta, buf.C_ref, ct, ldc, buf.sc, batch, comp)
    elif case.api == "gemm_batched_ex":
        ours = lambda: h.gemm_batched_ex(ta, tb, m, n, k, alpha, buf.Aarr, at, lda, buf.Barr, bt, ldb, beta,  # noqa
                                         buf.Carr_ours, ct, ldc, batch, comp)
        theirs = lambda: cb.gemm_batched_ex(ta, tb, m, n, k, alpha, buf.Aarr, at, lda, buf.Barr, bt, ldb,  # noqa
                                            beta, buf.Carr_ref, ct, ldc, batch, comp)
    else:
        raise ValueError(f"no runnable path for api {case.api}")
    return ours, theirs


def _time(fn, warmup: int, iters: int, check) -> float:
    for _ in range(warmup):
        check(fn())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        check(fn())
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / max(1, iters)


def _validate(case: mf.Case, buf: _Buffers) -> tuple[bool, float]:
    """Our C against cuBLAS's C on the same inputs: (ok, normwise relative difference)."""
    if case.c_type == mf.R32I:
        diff = int((buf.C_ours != buf.C_ref).sum().item())
        return diff == 0, float(diff)
    if case.c_type == mf.R16F:
        got = buf.C_ours.view(torch.float16).double()
        ref = buf.C_ref.view(torch.float16).double()
        tol = VALIDATION_TOL["f16_out"]
    else:
        got, ref = buf.C_ours.double(), buf.C_ref.double()
        tol = VALIDATION_TOL["f32"] if case.a_type == mf.R32F else VALIDATION_TOL["lowp"]
    if case.compute_type in (mf.F16, mf.F32_TF32):
        # cuBLAS may accumulate in f16 or multiply in TF32 for these compute types, while this backend
        # accumulates in f32 (FP16 inputs) or stays exact f32 (FAST_TF32): the reference side is the
        # less accurate one, so the bound is that of a 10-bit-mantissa computation.
        tol = VALIDATION_TOL["lowp"]
    den = float(torch.linalg.norm(ref)) or 1.0
    err = float(torch.linalg.norm(got - ref)) / den
    return err <= tol, err


def run_case(case: mf.Case, h: gs.Handle, cb: cublas_ref.Cublas, warmup: int, iters: int, device,
             scalar_fn=None) -> dict:
    """Times one runnable case; returns its row (status "ok" or "validation_failed" before the perf gates)."""
    buf = _Buffers(case, device)
    ours, theirs = _calls(case, h, cb, buf)

    def ok_status(s):
        if s != 0:
            raise RuntimeError(f"call failed with status {s}")

    cublas_ms = _time(theirs, warmup, iters, ok_status)
    shader_ms = _time(ours, warmup, iters, ok_status)
    # Results of a single call from the original C (beta = 0 makes them independent of the repeats).
    valid, err = _validate(case, buf)
    s, batch = case.shape, buf.batch
    row = mf.row_prefix(case, "ok" if valid else "validation_failed")
    scalar_ms = scalar_tf = None
    scalar_info = {}
    if scalar_fn is not None:
        r = scalar_fn(case)
        if r is not None:
            scalar_ms, (sm, sn, sk, sbatch) = r
            scalar_tf = tflops(sm, sn, sk, scalar_ms, sbatch)
            scalar_info = {"scalar_shape": [sm, sn, sk], "scalar_batch": sbatch, "scalar_cores": 1}
    row.update({"cublas_ms": round(cublas_ms, 6), "cublas_tflops": round(tflops(s.m, s.n, s.k, cublas_ms, batch), 4),
                "scalar_ms": None if scalar_ms is None else round(scalar_ms, 6),
                "scalar_tflops": None if scalar_tf is None else round(scalar_tf, 6),
                "shader_ms": round(shader_ms, 6), "shader_tflops": round(tflops(s.m, s.n, s.k, shader_ms, batch), 4),
                "shader_cublas_ratio": round(shader_ms / cublas_ms, 6) if cublas_ms > 0 else None})
    row.update({"batch_count": batch, "kernels": gs_kernel_names(h.last_kernels()),
                "validation": {"against": "cuBLAS", "metric": "mismatches" if case.c_type == mf.R32I else "normwise",
                               "value": err}})
    row.update(scalar_info)
    return row


def gs_kernel_names(bits: int) -> list[str]:
    names = [(gs.KERNEL_TC_F16, "tc_f16"), (gs.KERNEL_TC_BF16, "tc_bf16"), (gs.KERNEL_TC_I8, "tc_i8"),
             (gs.KERNEL_FFMA, "ffma_f32"), (gs.KERNEL_SIMT, "simt"), (gs.KERNEL_SCALE, "scale"),
             (gs.KERNEL_TMAP, "tmap_build"), (gs.KERNEL_TC_TF32, "tc_tf32"), (gs.KERNEL_REDUCE, "splitk_reduce")]
    return [n for b, n in names if bits & b]


# ---- the loop with summary (bench/gemm_perf.zig:50-89, :192-234) ----------------------------------------------
class Summary:
    def __init__(self):
        self.accelerated = 0
        self.log_ratio_sum = 0.0
        self.regressions = 0
        self.strict = 0
        self.strict_failures = 0
        self.strict_worst = 0.0

    def line(self) -> dict:
        geo = math.exp(self.log_ratio_sum / self.accelerated) if self.accelerated else None
        return {"summary": "hardware_accelerated", "cases": self.accelerated,
                "geomean_shader_cublas_ratio": None if geo is None else round(geo, 6),
                "regressions": self.regressions, "strict_cases": self.strict,
                "strict_failures": self.strict_failures, "strict_worst_ratio": round(self.strict_worst, 6)}

    def geomean(self):
        return math.exp(self.log_ratio_sum / self.accelerated) if self.accelerated else None


class Runner:
    def __init__(self, emit, warmup=5, iters=20, fail_every_row=False, only_cublas_supported=False,
                 tile_compatible_only=False, scalar_fn=None, device=None):
        self.emit = emit
        self.warmup, self.iters = warmup, iters
        self.fail_every_row = fail_every_row
        self.only_cublas_supported = only_cublas_supported
        self.tile_compatible_only = tile_compatible_only
        self.scalar_fn = scalar_fn
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.summary = Summary()
        self._h = None
        self._cb = None

    def _libs(self):
        if self._h is None:
            stream = torch.cuda.current_stream(self.device)
            self._h = gs.Handle(stream)
            self._cb = cublas_ref.Cublas(stream.cuda_stream)
        return self._h, self._cb

    def strict_unavailable(self, case: mf.Case) -> bool:
        if self.fail_every_row and case.cublas_supported() and not case.hardware_accelerated():
            self.summary.strict += 1
            self.summary.strict_failures += 1
            self.emit(mf.status_row(case, "shader_unavailable"))
            return True
        return False

    def run_case(self, case: mf.Case):
        """runCase (bench/gemm_perf.zig:192-234)."""
        if self.only_cublas_supported and not case.cublas_supported():
            return
        if self.tile_compatible_only and not case.tile_compatible():
            return
        if self.strict_unavailable(case):
            return
        status = case.base_status()
        if status != "ok":
            self.emit(mf.status_row(case, status))
            return
        h, cb = self._libs()
        row = run_case(case, h, cb, self.warmup, self.iters, self.device, self.scalar_fn)
        ratio = row["shader_cublas_ratio"]
        if row["status"] == "ok" and ratio is not None:
            final = "ok"
            if case.hardware_accelerated():
                self.summary.accelerated += 1
                self.summary.log_ratio_sum += math.log(ratio)
                if ratio > 1.0:
                    self.summary.regressions += 1
                    final = "perf_regression"
            if self.fail_every_row:
                self.summary.strict += 1
                self.summary.strict_worst = max(self.summary.strict_worst, ratio)
                if ratio >= 1.0:
                    self.summary.strict_failures += 1
                    final = "perf_regression"
            row["status"] = mf.STATUS_LABELS[final]
        self.emit(row)

    def run_manifest_case(self, case: mf.Case):
        """The --manifest=all enumeration body (bench/gemm_perf.zig:121-133)."""
        if self.tile_compatible_only and not case.tile_compatible():
            return
        if self.strict_unavailable(case):
            return
        if case.cublas_supported() and case.dispatch_available():
            self.run_case(case)
            return
        if self.only_cublas_supported and not case.cublas_supported():
            return
        self.emit(mf.status_row(case, case.base_status()))

    def run(self, sizes, rect_shapes, manifest_all: bool):
        if manifest_all:
            for size in sizes:
                for case in mf.compact_cases(mf.Shape(size, size, size)):
                    self.run_case(case)
            for shape in rect_shapes:
                for case in mf.compact_cases(shape):
                    self.run_case(case)
            side = sizes[0] if (self.tile_compatible_only and sizes) else 128
            for case in mf.manifest_cases(mf.Shape(side, side, side)):
                self.run_manifest_case(case)
        else:
            for size in sizes:
                self.run_case(mf.Case("regular", "N", "N", mf.R32F, mf.R32F, mf.R32F, mf.F32,
                                      mf.Shape(size, size, size)))
        self.emit(self.summary.line())
        return self.summary
