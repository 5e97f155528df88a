"""The Zig drop-in for slang-gemm's src/vulkan_runner.zig (slang-gemm_b200/zig/cuda_runner.zig).

Zig is not installed here, so the file cannot be compiled; these CPU tests check what the unmodified
bench/gemm_perf.zig needs from it, against the reference's interface (tests/golden/vulkan_runner_api.json,
made by make_vulkan_runner_api.py from the reference sources, and re-read from the reference itself when
it is present):
  * every `vulkan_runner.<name>` the bench uses is exported, with the reference runner's parameter list;
  * every other public bench* function of the reference runner is exported with its parameter list;
  * `Result` has the reference's fields, and the error set holds every error name the bench's catch
    switches list (a switch prong naming an error outside the set does not compile);
  * every gs_* function and GS_* constant the file uses is declared in include/gemm_sm100.h, and each
    gs_* call passes as many arguments as the header declares;
  * the library exports gs_select_device, and without a GPU it answers "no device" as the runner expects.
"""
import json
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ZIG = os.path.join(ROOT, "slang-gemm_b200", "zig", "cuda_runner.zig")
HEADER = os.path.join(ROOT, "include", "gemm_sm100.h")
FIXTURE = os.path.join(ROOT, "tests", "golden", "vulkan_runner_api.json")
REFERENCE = "/root/reference"


def _src() -> str:
    return open(ZIG).read()


def _api() -> dict:
    return json.load(open(FIXTURE))


def _exports(src: str) -> dict:
    return {name: " ".join(params.split()) for name, params in re.findall(r"^pub fn (\w+)\(([^)]*)\)", src, re.M)}


def _split_args(text: str) -> list:
    """Top-level comma split of a call's argument text."""
    out, depth, cur = [], 0, ""
    for ch in text:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur)
    return out


def _calls(src: str, name: str) -> list:
    """Argument lists of every `c.<name>(...)` call in src."""
    res = []
    for m in re.finditer(r"\bc\." + name + r"\(", src):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        res.append(_split_args(src[m.end():i - 1]))
    return res


def _header_decls() -> dict:
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return {name: _split_args(params) for name, params in re.findall(r"\b(gs_\w+)\s*\(([^;{]*?)\)\s*;", text)}


def test_fixture_matches_the_reference_sources():
    if not os.path.isdir(REFERENCE):
        pytest.skip("reference sources not present")
    import sys

    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_vulkan_runner_api as mk

    assert mk.extract(REFERENCE) == _api()


def test_every_runner_function_the_bench_calls_is_exported_with_its_signature():
    api, exp = _api(), _exports(_src())
    calls = [c for c in api["bench_calls"] if c != "Result"]
    assert len(calls) == 11
    for name in calls:
        assert name in exp, f"cuda_runner.zig does not export {name}"
        assert exp[name] == api["signatures"][name], name


def test_every_public_bench_function_of_the_reference_runner_is_exported():
    api, exp = _api(), _exports(_src())
    for name, params in api["signatures"].items():
        assert exp.get(name) == params, name


def test_result_type_and_error_set_fit_the_bench():
    src, api = _src(), _api()
    m = re.search(r"pub const Result = struct \{([^}]*)\}", src)
    assert m and [list(f) for f in re.findall(r"(\w+):\s*(\w+)", m.group(1))] == api["result_fields"]
    e = re.search(r"pub const Error = error\{([^}]*)\}", src)
    members = set(re.findall(r"(\w+)", e.group(1)))
    assert set(api["catch_errors"]) <= members
    # every exported bench* function returns that error set
    for name, ret in re.findall(r"^pub fn (bench\w*)\([^)]*\) (\S+) \{", src, re.M):
        assert ret == "Error!?Result", name


def test_library_calls_match_the_header():
    src, decls = _src(), _header_decls()
    assert '@cImport(@cInclude("gemm_sm100.h"))' in src
    used = set(re.findall(r"\bc\.(gs_\w+)\(", src))
    assert used >= {"gs_select_device", "gs_create", "gs_destroy", "gs_gemm_strided_batched_ex", "gs_device_error"}
    for name in used:
        assert name in decls, f"{name} is not declared in include/gemm_sm100.h"
        for args in _calls(src, name):
            assert len(args) == len(decls[name]), f"{name}: {len(args)} arguments, header declares {len(decls[name])}"
    header = open(HEADER).read()
    for const in set(re.findall(r"\bc\.(GS_\w+)", src)):
        assert re.search(r"\b" + const + r"\b\s*=", header), f"{const} is not defined in include/gemm_sm100.h"


def test_select_device_is_exported_and_reports_no_device_without_a_gpu():
    import gemm_sm100 as gs

    assert "gs_select_device" in gs.declared_symbols()
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    status, dev = gs.select_device(None)
    assert status == gs.STATUS_NOT_INITIALIZED and dev == -1
    status, _ = gs.select_device("B200")
    assert status == gs.STATUS_NOT_INITIALIZED


def test_library_call_wrappers_take_cublas_zig_arguments():
    import sys

    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_vulkan_runner_api as mk

    src = _src()
    assert re.search(r"^pub const Context = struct \{", src, re.M)
    ours = {name: mk.param_types(params) for name, params in re.findall(r"^pub fn (\w+)\(([^)]*)\)", src, re.M)}
    for name, types in _api()["cublas_calls"].items():
        # RawGemmExDesc / RawGemmBatchedExDesc are the reference's own descriptors, used as they are
        expect = [("cublas." + t if t.startswith("Raw") else t) for t in types]
        assert ours.get(name) == expect, name


@pytest.mark.gpu
def test_select_device_picks_a_b200_by_name(cuda):
    import gemm_sm100 as gs

    status, dev = gs.select_device(None)
    assert status == gs.STATUS_SUCCESS and dev >= 0
    status, dev2 = gs.select_device("B200")
    assert status == gs.STATUS_SUCCESS and dev2 >= 0
    status, _ = gs.select_device("no-such-device-name")
    assert status == gs.STATUS_INVALID_VALUE
