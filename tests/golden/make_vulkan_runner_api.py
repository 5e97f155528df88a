"""Writes vulkan_runner_api.json: the interface of slang-gemm's src/vulkan_runner.zig that
bench/gemm_perf.zig depends on, read from the reference sources.

  bench_calls     every `vulkan_runner.<name>` the bench uses (names, sorted)
  signatures      parameter list of every `pub fn bench*` in src/vulkan_runner.zig
  catch_errors    every error name the bench's `catch |err| switch (err)` prongs list
  result_fields   the fields of vulkan_runner.Result
  cublas_calls    parameter types of the src/cublas.zig library calls the runner mirrors

Run from the repository root: python tests/golden/make_vulkan_runner_api.py [REFERENCE_ROOT]
"""
import json
import os
import re
import sys


def extract(ref: str) -> dict:
    bench = open(os.path.join(ref, "bench", "gemm_perf.zig")).read()
    runner = open(os.path.join(ref, "src", "vulkan_runner.zig")).read()
    calls = sorted(set(re.findall(r"\bvulkan_runner\.(\w+)", bench)))
    sigs = {name: " ".join(params.split())
            for name, params in re.findall(r"^pub fn (bench\w*)\(([^)]*)\)", runner, re.M)}
    errors = set()
    for prong in re.findall(r"catch \|err\| switch \(err\) \{\s*([^=]*)=> null", bench):
        errors.update(re.findall(r"error\.(\w+)", prong))
    m = re.search(r"pub const Result = struct \{([^}]*)\}", runner)
    fields = re.findall(r"(\w+):\s*(\w+)", m.group(1)) if m else []
    cub = open(os.path.join(ref, "src", "cublas.zig")).read()
    mirrored = ("sgemm", "sgemmStridedBatched", "sgemmBatched", "gemmEx", "gemmStridedBatchedEx", "gemmBatchedEx")
    cublas_calls = {name: param_types(params) for name, params in re.findall(r"^pub fn (\w+)\(([^)]*)\)", cub, re.M)
                    if name in mirrored}
    return {"bench_calls": calls, "signatures": sigs, "catch_errors": sorted(errors),
            "result_fields": [list(f) for f in fields], "cublas_calls": cublas_calls}


def param_types(params: str) -> list:
    """Types of a Zig parameter list, without the names (\"a: T, b: U\" -> [\"T\", \"U\"])."""
    return [p.split(":", 1)[1].strip() for p in params.split(",") if ":" in p]


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "vulkan_runner_api.json")
    with open(out, "w") as f:
        json.dump(extract(ref), f, indent=1, sort_keys=True)
        f.write("\n")
    print(out)
