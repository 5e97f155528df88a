"""Manifest case model and benchmark-row logic on the CPU (no GPU calls).

Mirrors slang-gemm's tests/gemm_manifest.zig (predicates and labels of
src/manifest.zig) for this backend, checks that the manifest's dispatch
claims agree with the library's own planner, and exercises the row / summary
logic of bench/gemm_perf.zig on status-only rows.
"""
import json

import numpy as np
import pytest

import gemm_sm100 as gs
import manifest as mf
import oracle as orc
import perf_rows as pr

SHAPE = mf.Shape(128, 128, 128)
TENSOR_SHAPE = mf.Shape(256, 256, 256)


def test_runnable_fp32_case():
    """tests/gemm_manifest.zig:8-27."""
    case = mf.Case("regular", "N", "N", mf.R32F, mf.R32F, mf.R32F, mf.F32, SHAPE)
    assert case.cublas_supported() and case.shader_implemented() and case.dispatch_available()
    assert case.base_status() == "ok"
    assert case.family() == "classic_sgemm"
    assert case.shader_family() == "f32_tf32"
    assert not case.hardware_accelerated()          # FFMA, not the tensor cores


def test_tensor_ex_case():
    """tests/gemm_manifest.zig:29-49."""
    case = mf.Case("gemm_ex", "N", "N", mf.R16F, mf.R16F, mf.R32F, mf.F32, TENSOR_SHAPE)
    assert case.cublas_supported() and case.shader_implemented() and case.hardware_accelerated()
    assert case.tile_compatible() and case.dispatch_available()
    assert case.base_status() == "ok"
    assert case.family() == "tensor_ex"
    assert case.shader_family() == "f16_bf16_tensor"


def test_tile_compatibility():
    """tests/gemm_manifest.zig:51-77."""
    ok = mf.Case("gemm_ex", "N", "N", mf.R16F, mf.R16F, mf.R32F, mf.F32, mf.Shape(256, 256, 256))
    no = mf.Case("gemm_ex", "N", "N", mf.R16F, mf.R16F, mf.R32F, mf.F32, mf.Shape(256, 128, 256))
    assert ok.tile_compatible() and not no.tile_compatible()
    # this backend's tensor-core kernels take ragged shapes: the tile filter is not an acceleration gate
    assert no.hardware_accelerated()


def test_unsupported_enum_combination_and_labels():
    """tests/gemm_manifest.zig:79-96."""
    case = mf.Case("gemm_ex", "N", "N", "CUDA_R_4F_E2M1", "CUDA_R_4F_E2M1", mf.R32F, mf.F32, SHAPE)
    assert not case.cublas_supported() and not case.shader_implemented()
    assert case.base_status() == "cublas_unsupported"
    assert mf.STATUS_LABELS[case.base_status()] == "cuBLAS_unsupported"
    assert mf.DATA_TYPES["CUDA_R_4F_E2M1"] == 33 and mf.COMPUTE_TYPES["CUBLAS_COMPUTE_32F"] == 68
    assert mf.OPS == ["N", "T", "C"]


def test_enum_values_match_the_library():
    assert mf.DATA_TYPES[mf.R16F] == gs.R_16F and mf.DATA_TYPES[mf.R16BF] == gs.R_16BF
    assert mf.DATA_TYPES[mf.R8I] == gs.R_8I and mf.DATA_TYPES[mf.R32I] == gs.R_32I
    assert mf.COMPUTE_TYPES[mf.F32_TF32] == gs.COMPUTE_32F_FAST_TF32 and mf.COMPUTE_TYPES[mf.I32] == gs.COMPUTE_32I


@pytest.mark.parametrize("api,op_a,op_b,a,c,comp", [
    ("regular", "N", "N", mf.R32F, mf.R32F, mf.F32),
    ("gemm_ex", "N", "N", mf.R16F, mf.R16F, mf.F16),
    ("gemm_ex", "T", "N", mf.R16F, mf.R32F, mf.F32_16F),
    ("gemm_ex", "N", "T", mf.R16BF, mf.R32F, mf.F32_16BF),
    ("gemm_ex", "C", "N", mf.R32F, mf.R32F, mf.F32_TF32),
    ("gemm_ex", "N", "C", mf.R8I, mf.R32I, mf.I32),
    ("gemm_strided_batched_ex", "N", "N", mf.R16F, mf.R32F, mf.F32),
])
def test_compact_families_dispatch(api, op_a, op_b, a, c, comp):
    """tests/gemm_manifest.zig:98-122, restricted to this backend's (real, non-FP64) families."""
    case = mf.Case(api, op_a, op_b, a, a, c, comp, SHAPE, api in mf.BATCHED_APIS)
    assert case.cublas_supported() and case.shader_implemented() and case.shader_family() != "none"


def test_only_fp64_and_complex_are_unavailable():
    """tests/gemm_manifest.zig:124-161 for this backend: of the cuBLAS-supported manifest, only the FP64 and complex
    rows (out of this backend's scope) lack a kernel."""
    for case in mf.manifest_cases(SHAPE):
        if not case.cublas_supported():
            continue
        wide = case.a_type in (mf.R64F, mf.C32F, mf.C64F) or case.api == "complex_3m"
        assert case.dispatch_available() == (not wide), case
        assert case.base_status() == ("shader_unavailable" if wide else "ok")


def test_dispatch_claims_match_planner_statuses():
    """Every Ex case the manifest dispatches is accepted by gs_plan_gemm_strided_batched_ex, and every Ex case it
    does not dispatch is refused with NOT_SUPPORTED."""
    seen = 0
    for case in mf.manifest_cases(SHAPE):
        if case.api not in mf.EX_APIS:
            continue
        st, _ = mf.plan_kernel(case)
        if case.dispatch_available():
            assert st == gs.STATUS_SUCCESS, case
            seen += 1
        elif case.cublas_supported():
            assert st != gs.STATUS_SUCCESS, case
    assert seen > 50


def test_kernel_families_of_accelerated_rows():
    tc = [c for c in mf.manifest_cases(TENSOR_SHAPE) if c.hardware_accelerated()]
    assert tc and all(c.a_type in (mf.R16F, mf.R16BF, mf.R8I) for c in tc)
    assert not any(c.a_type == mf.R32F for c in tc)


def test_fills_follow_the_reference_bench():
    """fill / fillI8 (bench/gemm_perf.zig:1184-1189, :1239-1244) against the oracle's copies of the same formulas;
    the f16 conversion agrees with round-to-nearest-even except on exact ties."""
    f = pr.fill_f32(4096, 0.1)
    assert np.allclose(f, orc.value_for(np.arange(4096), 0.1).astype(np.float32), atol=1e-6)
    assert np.array_equal(pr.fill_i8(1000, 1), orc.fill_i8(1000, 1))
    bits = pr.fill_lowp16(4096, mf.R16F, -0.2)
    rne = np.array([orc.f32_to_f16_bits(float(v)) for v in pr.fill_f32(4096, -0.2)], np.uint16)
    assert (bits != rne).sum() <= 4096 // 23 + 1
    bf = pr.fill_lowp16(64, mf.R16BF, 0.1)
    assert np.array_equal(bf, (pr.fill_f32(64, 0.1).view(np.uint32) >> 16).astype(np.uint16))


def _runner(**kw):
    rows = []
    return rows, pr.Runner(rows.append, device="cpu", **kw)


def test_status_rows_and_summary_without_runnable_cases():
    rows, r = _runner()
    r.run_case(mf.Case("gemm_ex", "N", "N", "CUDA_R_4F_E2M1", "CUDA_R_4F_E2M1", mf.R32F, mf.F32, SHAPE))
    r.run_case(mf.Case("regular", "N", "N", mf.R64F, mf.R64F, mf.R64F, mf.F64, SHAPE))
    assert [x["status"] for x in rows] == ["cuBLAS_unsupported", "shader_unavailable"]
    assert all(x[k] is None for x in rows for k in mf.TIMING_KEYS)
    assert list(rows[0])[:16] == ["status", "api", "family", "shader_family", "shader_implemented",
                                  "dispatch_available", "op_a", "op_b", "a_type", "b_type", "c_type",
                                  "compute_type", "m", "n", "k", "cublas_ms"]
    assert r.summary.line() == {"summary": "hardware_accelerated", "cases": 0, "geomean_shader_cublas_ratio": None,
                                "regressions": 0, "strict_cases": 0, "strict_failures": 0, "strict_worst_ratio": 0.0}
    json.dumps(rows)


def test_fail_every_row_marks_non_tensor_rows():
    """--fail-every-row: a cuBLAS-supported row off the tensor cores is a strict failure (bench/gemm_perf.zig:195-199)."""
    rows, r = _runner(fail_every_row=True)
    r.run_case(mf.Case("regular", "N", "N", mf.R32F, mf.R32F, mf.R32F, mf.F32, SHAPE))
    assert rows[0]["status"] == "shader_unavailable"
    assert r.summary.strict == 1 and r.summary.strict_failures == 1


def test_filters_skip_rows():
    rows, r = _runner(only_cublas_supported=True, tile_compatible_only=True)
    r.run_case(mf.Case("gemm_ex", "N", "N", "CUDA_R_4F_E2M1", "CUDA_R_4F_E2M1", mf.R32F, mf.F32, SHAPE))
    r.run_case(mf.Case("gemm_ex", "N", "N", mf.R16F, mf.R16F, mf.R32F, mf.F32, mf.Shape(100, 128, 128)))
    assert rows == []


def test_manifest_enumeration_size():
    cases = list(mf.manifest_cases(SHAPE))
    assert len(cases) == len(mf.APIS) * 9 * (len(mf.DATA_TYPES) * len(mf.COMPUTE_TYPES) + 4)
    compact = list(mf.compact_cases(SHAPE))
    assert len(compact) == 9 + 9
