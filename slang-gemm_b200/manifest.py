"""Case model of the benchmark manifest: which API / op / type / compute-type
combinations exist, which of them cuBLAS supports, which this backend
dispatches, and the JSONL labels of each row.

Restates slang-gemm's src/manifest.zig for the CUDA backend:
  - Api, Status and ShaderFamily labels: src/manifest.zig:4-73;
  - Case.family / cublasSupported / tileCompatible / baseStatus:
    src/manifest.zig:80-205, exTypeSupported :404-410;
  - the enumerated apis / ops / data types / compute types and their labels:
    src/manifest.zig:214-343; default shapes :345-358.
The JSON keys keep the reference's names ("shader_family", "shader_ms", ...)
so rows stay comparable; "shader" means this backend's CUDA kernels.

What differs, because the backend differs: dispatch_available is what
libgemm_sm100 computes (FP32 classic and Ex, FP16 / BF16 -> FP32 or same
type, INT8 -> INT32; no FP64, complex or packed low-precision types), and
hardware_accelerated asks the library's own planner whether the case runs on
the tcgen05 tensor-core kernels (gs_plan_gemm_strided_batched_ex), instead of
the reference's per-shader tile predicates.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import gemm_sm100 as gs

# ---- enums with the reference's label strings ------------------------------------------------------------------
APIS = ["regular", "regular_64", "batched", "strided_batched", "complex_3m", "gemm_ex", "gemm_batched_ex",
        "gemm_strided_batched_ex"]
EX_APIS = ("gemm_ex", "gemm_batched_ex", "gemm_strided_batched_ex")
CLASSIC_APIS = ("regular", "regular_64", "batched", "strided_batched")
BATCHED_APIS = ("batched", "strided_batched", "gemm_batched_ex", "gemm_strided_batched_ex")

OPS = ["N", "T", "C"]
OP_VALUE = {"N": gs.OP_N, "T": gs.OP_T, "C": gs.OP_C}

# cudaDataType names with their CUDA integer values (src/gemm.zig:14-49).
DATA_TYPES = {
    "CUDA_R_16F": 2, "CUDA_C_16F": 6, "CUDA_R_16BF": 14, "CUDA_C_16BF": 15, "CUDA_R_32F": 0, "CUDA_C_32F": 4,
    "CUDA_R_64F": 1, "CUDA_C_64F": 5, "CUDA_R_4I": 16, "CUDA_C_4I": 17, "CUDA_R_4U": 18, "CUDA_C_4U": 19,
    "CUDA_R_8I": 3, "CUDA_C_8I": 7, "CUDA_R_8U": 8, "CUDA_C_8U": 9, "CUDA_R_16I": 20, "CUDA_C_16I": 21,
    "CUDA_R_16U": 22, "CUDA_C_16U": 23, "CUDA_R_32I": 10, "CUDA_C_32I": 11, "CUDA_R_32U": 12, "CUDA_C_32U": 13,
    "CUDA_R_64I": 24, "CUDA_C_64I": 25, "CUDA_R_64U": 26, "CUDA_C_64U": 27, "CUDA_R_8F_E4M3": 28,
    "CUDA_R_8F_E5M2": 29, "CUDA_R_8F_UE8M0": 30, "CUDA_R_6F_E2M3": 31, "CUDA_R_6F_E3M2": 32, "CUDA_R_4F_E2M1": 33,
}
# cublasComputeType_t names with their values (src/gemm.zig:53-67).
COMPUTE_TYPES = {
    "CUBLAS_COMPUTE_16F": 64, "CUBLAS_COMPUTE_16F_PEDANTIC": 65, "CUBLAS_COMPUTE_32F": 68,
    "CUBLAS_COMPUTE_32F_PEDANTIC": 69, "CUBLAS_COMPUTE_32F_FAST_16F": 74, "CUBLAS_COMPUTE_32F_FAST_16BF": 75,
    "CUBLAS_COMPUTE_32F_FAST_TF32": 77, "CUBLAS_COMPUTE_32F_EMULATED_16BFX9": 78, "CUBLAS_COMPUTE_64F": 70,
    "CUBLAS_COMPUTE_64F_PEDANTIC": 71, "CUBLAS_COMPUTE_64F_EMULATED_FIXEDPOINT": 79, "CUBLAS_COMPUTE_32I": 72,
    "CUBLAS_COMPUTE_32I_PEDANTIC": 73,
}

R16F, R16BF, R32F, R64F, C32F, C64F, R8I, R32I = ("CUDA_R_16F", "CUDA_R_16BF", "CUDA_R_32F", "CUDA_R_64F",
                                                  "CUDA_C_32F", "CUDA_C_64F", "CUDA_R_8I", "CUDA_R_32I")
F16, F32, F32P, F32_16F, F32_16BF, F32_TF32, F64, I32, I32P = (
    "CUBLAS_COMPUTE_16F", "CUBLAS_COMPUTE_32F", "CUBLAS_COMPUTE_32F_PEDANTIC", "CUBLAS_COMPUTE_32F_FAST_16F",
    "CUBLAS_COMPUTE_32F_FAST_16BF", "CUBLAS_COMPUTE_32F_FAST_TF32", "CUBLAS_COMPUTE_64F", "CUBLAS_COMPUTE_32I",
    "CUBLAS_COMPUTE_32I_PEDANTIC")

STATUS_LABELS = {"ok": "ok", "cublas_unsupported": "cuBLAS_unsupported", "shader_unavailable": "shader_unavailable",
                 "validation_failed": "validation_failed", "perf_regression": "perf_regression",
                 "invalid": "invalid"}
FAMILY_LABELS = {"none": "none", "f16_scalar": "gemm_family_f16_scalar",
                 "f16_bf16_tensor": "gemm_family_f16_bf16_tensor", "f32_tf32": "gemm_family_f32_tf32",
                 "f64": "gemm_family_f64", "complex_f32": "gemm_family_complex_f32",
                 "complex_f64": "gemm_family_complex_f64", "int8_int32": "gemm_family_int8_int32",
                 "low_precision_f32": "gemm_family_low_precision_packed"}
LOW_PRECISION = (R16F, R16BF, "CUDA_R_8F_E4M3", "CUDA_R_8F_E5M2", "CUDA_R_8F_UE8M0", "CUDA_R_6F_E2M3",
                 "CUDA_R_6F_E3M2", "CUDA_R_4F_E2M1")


@dataclass(frozen=True)
class Shape:
    m: int
    n: int
    k: int


DEFAULT_SHAPES = [Shape(128, 128, 128), Shape(256, 256, 256), Shape(512, 512, 512), Shape(1024, 1024, 1024),
                  Shape(2048, 2048, 2048), Shape(4096, 4096, 4096), Shape(256, 512, 128), Shape(512, 256, 1024),
                  Shape(1024, 4096, 512), Shape(4096, 1024, 2048)]


def _classic_type(a, b, c):
    return (a, b, c) in ((R32F,) * 3, (R64F,) * 3, (C32F,) * 3, (C64F,) * 3)


def _classic_compute(a, comp):
    if a in (R32F, C32F):
        return comp == F32
    if a in (R64F, C64F):
        return comp == F64
    return False


def ex_type_supported(a, b, c, comp) -> bool:
    """exTypeSupported (src/manifest.zig:404-410): the cuBLAS gemmEx combinations the manifest tracks."""
    if a == b == c == R32F and comp in (F32, F32_TF32, F32P):
        return True
    if a == b == R16F and c in (R16F, R32F) and comp in (F16, F32, F32_16F):
        return True
    if a == b == R16BF and c == R32F and comp in (F32, F32_16BF):
        return True
    if a == b == R8I and c == R32I and comp in (I32, I32P):
        return True
    return False


@dataclass(frozen=True)
class Case:
    api: str
    op_a: str
    op_b: str
    a_type: str
    b_type: str
    c_type: str
    compute_type: str
    shape: Shape
    batched: bool = field(default=False)

    # ---- restated predicates (src/manifest.zig:80-205) ----
    def family(self) -> str:
        t = (self.a_type, self.b_type, self.c_type)
        if self.api == "regular":
            for name, ty in (("classic_sgemm", R32F), ("classic_dgemm", R64F), ("classic_cgemm", C32F),
                             ("classic_zgemm", C64F)):
                if t == (ty,) * 3:
                    return name
        if self.api in EX_APIS:
            if (self.a_type == self.b_type and self.a_type in (R16F, R16BF)) or \
                    (self.a_type == self.b_type == R32F and self.compute_type == F32_TF32):
                return "tensor_ex"
            if self.a_type == self.b_type == R8I and self.compute_type == I32:
                return "int8_ex"
        return "generic"

    def cublas_supported(self) -> bool:
        if self.api in CLASSIC_APIS:
            return _classic_type(self.a_type, self.b_type, self.c_type) and _classic_compute(self.a_type,
                                                                                             self.compute_type)
        if self.api == "complex_3m":
            return (self.a_type, self.b_type, self.c_type, self.compute_type) in ((C32F, C32F, C32F, F32),
                                                                                  (C64F, C64F, C64F, F64))
        return ex_type_supported(self.a_type, self.b_type, self.c_type, self.compute_type)

    def shader_family(self) -> str:
        if not self.cublas_supported():
            return "none"
        a, b, c = self.a_type, self.b_type, self.c_type
        if self.api in CLASSIC_APIS:
            return {R32F: "f32_tf32", R64F: "f64", C32F: "complex_f32", C64F: "complex_f64"}[a]
        if self.api == "complex_3m":
            return "complex_f32" if a == C32F else "complex_f64"
        if a == b == c == R32F:
            return "f32_tf32"
        if a == b == c == R16F:
            return "f16_scalar"
        if a == b and a in (R16F, R16BF) and c == R32F:
            return "f16_bf16_tensor"
        if a == b == R8I and c == R32I:
            return "int8_int32"
        if a in LOW_PRECISION and b in LOW_PRECISION and c == R32F:
            return "low_precision_f32"
        return "none"

    def shader_implemented(self) -> bool:
        """A CUDA kernel family of this backend computes the case (FP64 / complex are out of its scope)."""
        return self.dispatch_available()

    def tile_compatible(self) -> bool:
        """tileCompatible (src/manifest.zig:180-198), kept as the reference's shape filter."""
        if not self.cublas_supported():
            return False
        s, a, b, c = self.shape, self.a_type, self.b_type, self.c_type
        if a == b == R16F and c == R32F:
            return s.m % 128 == 0 and s.n % 256 == 0 and s.k % 16 == 0
        if a == b == R16BF and c == R32F:
            return s.m % 64 == 0 and s.n % 128 == 0 and s.k % 16 == 0
        if a == b == R8I and c == R32I:
            return s.m % 128 == 0 and s.n % 256 == 0 and s.k % 32 == 0
        if a in (R32F, C32F):
            return s.m % 64 == 0 and s.n % 64 == 0 and s.k % 16 == 0
        if a in (R64F, C64F):
            return s.m % 32 == 0 and s.n % 32 == 0 and s.k % 16 == 0
        return s.m % 16 == 0 and s.n % 16 == 0 and s.k % 16 == 0

    # ---- this backend ----
    def type_codes(self) -> tuple[int, int, int, int]:
        return (DATA_TYPES[self.a_type], DATA_TYPES[self.b_type], DATA_TYPES[self.c_type],
                COMPUTE_TYPES[self.compute_type])

    def dispatch_available(self) -> bool:
        """libgemm_sm100 has an entry point and a kernel for the case (checked through its planner)."""
        if not self.cublas_supported():
            return False
        if self.api == "complex_3m":
            return False
        if self.api in CLASSIC_APIS:
            return self.a_type == R32F and self.compute_type == F32
        return plan_kernel(self)[0] == gs.STATUS_SUCCESS

    def hardware_accelerated(self) -> bool:
        """The case runs on the tcgen05 tensor-core kernels (the rows the performance gate applies to)."""
        if not self.dispatch_available() or self.api in CLASSIC_APIS:
            return False
        st, kernel = plan_kernel(self)
        return st == gs.STATUS_SUCCESS and bool(kernel & (gs.KERNEL_TC_F16 | gs.KERNEL_TC_BF16 | gs.KERNEL_TC_I8))

    def base_status(self) -> str:
        if not self.cublas_supported():
            return "cublas_unsupported"
        if not self.dispatch_available():
            return "shader_unavailable"
        return "ok"

    def batch_count(self) -> int:
        """Batch entries a batched row times (4, as bench/gemm_perf.zig:1003-1015)."""
        return 4 if self.api in BATCHED_APIS else 1


_ALIGNED = 1 << 20  # stand-in 16-byte-aligned addresses for the pure-host planner


def plan_kernel(case: Case) -> tuple[int, int]:
    """(status, kernel bit) the library would use for the case with tight, aligned column-major operands."""
    a, b, c, comp = case.type_codes()
    s = case.shape
    opa, opb = OP_VALUE[case.op_a], OP_VALUE[case.op_b]
    lda = s.m if opa == gs.OP_N else s.k
    ldb = s.k if opb == gs.OP_N else s.n
    batch = case.batch_count()
    return gs.plan_gemm(opa, opb, s.m, s.n, s.k, _ALIGNED, a, max(1, lda), s.m * s.k, _ALIGNED * 2, b, max(1, ldb),
                        s.k * s.n, _ALIGNED * 4, c, max(1, s.m), s.m * s.n, batch, comp)


def manifest_cases(shape: Shape):
    """The --manifest=all enumeration for one shape (bench/gemm_perf.zig:104-158): every API x op x op over
    every data type as same-type rows, then the mixed tensor / integer rows."""
    for api in APIS:
        for op_a in OPS:
            for op_b in OPS:
                for dt in DATA_TYPES:
                    for comp in COMPUTE_TYPES:
                        yield Case(api, op_a, op_b, dt, dt, dt, comp, shape, api in BATCHED_APIS)
                for a, c, comp in ((R16F, R32F, F32), (R16BF, R32F, F32), (R32F, R32F, F32_TF32), (R8I, R32I, I32)):
                    yield Case(api, op_a, op_b, a, a, c, comp, shape, api in BATCHED_APIS)


def compact_cases(shape: Shape):
    """runCompactCasesForShape (bench/gemm_perf.zig:162-190)."""
    for op_a in OPS:
        for op_b in OPS:
            yield Case("regular", op_a, op_b, R32F, R32F, R32F, F32, shape)
    yield Case("regular", "T", "N", R64F, R64F, R64F, F64, shape)
    yield Case("regular", "C", "N", C32F, C32F, C32F, F32, shape)
    yield Case("regular", "N", "C", C64F, C64F, C64F, F64, shape)
    yield Case("complex_3m", "N", "N", C32F, C32F, C32F, F32, shape)
    yield Case("gemm_ex", "N", "N", R16F, R16F, R32F, F32, shape)
    yield Case("gemm_ex", "N", "N", R16BF, R16BF, R32F, F32, shape)
    yield Case("gemm_ex", "N", "N", R8I, R8I, R32I, I32, shape)
    yield Case("gemm_strided_batched_ex", "N", "N", R16F, R16F, R32F, F32, shape, True)
    yield Case("gemm_batched_ex", "N", "N", R16F, R16F, R32F, F32, shape, True)


def row_prefix(case: Case, status: str) -> dict:
    """The leading JSONL fields of a row (bench/gemm_perf.zig:224-228)."""
    return {"status": STATUS_LABELS[status], "api": case.api, "family": case.family(),
            "shader_family": FAMILY_LABELS[case.shader_family()], "shader_implemented": case.shader_implemented(),
            "dispatch_available": case.dispatch_available(), "op_a": case.op_a, "op_b": case.op_b,
            "a_type": case.a_type, "b_type": case.b_type, "c_type": case.c_type,
            "compute_type": case.compute_type, "m": case.shape.m, "n": case.shape.n, "k": case.shape.k}


TIMING_KEYS = ("cublas_ms", "cublas_tflops", "scalar_ms", "scalar_tflops", "shader_ms", "shader_tflops",
               "shader_cublas_ratio")


def status_row(case: Case, status: str) -> dict:
    """emitStatusOnly (bench/gemm_perf.zig:236-244): a row without timings."""
    row = row_prefix(case, status)
    row.update({k: None for k in TIMING_KEYS})
    return row
