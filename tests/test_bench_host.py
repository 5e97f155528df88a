"""Host-side logic of bench.py on the CPU: workload arithmetic, roofline bound
selection, the rank split, the committed profile lookups, the manifest scalar
column against the oracle, and the no-GPU paths of the CLI.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402
import manifest as mf  # noqa: E402

PEAKS = {"hbm_gbs": 6463.7, "bf16": 1667.5, "bf16_sustained": 1396.4, "sm_max_mhz": 1965.0, "source": "measured"}


def test_work_counts_flops_and_bytes():
    c3 = bench.CONFIGS["c3-f16-nn"]
    flops, byts = bench.work(c3)
    assert flops == 2.0 * 8192 ** 3
    assert byts == 8192 * 8192 * (2 + 2 + 4)          # A, B f16 + C f32 written once (beta = 0)
    c2 = bench.CONFIGS["c2-sgemm-nn"]                 # beta = 0.5: C read and written
    assert bench.work(c2)[1] == 4096 * 2048 * 4 + 2048 * 1024 * 4 + 4096 * 1024 * 4 * 2


@pytest.mark.parametrize("name,bound", [("c3-f16-nn", "tensor"), ("c5-i8-nn", "tensor"), ("c4-f16-strided", "hbm"),
                                        ("c2-sgemm-nn", "ffma"), ("c5b-i8-strided", "tensor")])
def test_roofline_bound_per_config(name, bound):
    cfg = bench.CONFIGS[name]
    flops, byts = bench.work(cfg)
    r = bench.roofline_of(cfg, flops, byts, 1.0, PEAKS, None)
    assert r["bound"] == bound
    assert 0 < r["frac"] and abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    if name == "c5-i8-nn":
        assert r["peak"] == pytest.approx(2 * PEAKS["bf16"])


def test_rank_share_weak_and_strong():
    c3 = bench.CONFIGS["c3-f16-nn"]
    weak, _ = bench.rank_share(c3, 1, 4, "weak")
    assert weak["n"] == 8192 and weak["m"] == 8192          # every rank holds a full configuration's work
    strong = [bench.rank_share(c3, r, 4, "strong")[0]["n"] for r in range(4)]
    assert sum(strong) == 8192 and all(x % 256 == 0 for x in strong)
    c4 = bench.CONFIGS["c4-f16-strided"]
    assert sum(bench.rank_share(c4, r, 8, "strong")[0]["batch"] for r in range(8)) == 256


def test_committed_profiles_cover_the_tensor_configs():
    for name in ("c3-f16-nn", "c3-bf16-nn", "c5-i8-nn", "c4-f16-strided", "c5b-i8-strided"):
        t = bench.committed_traffic(name)
        u = bench.committed_pipe_utilization(name)
        assert t is None or t > 0
        if u is not None:
            assert u["pipe"] in ("tensor", "FMA") and 0 < u["pct_of_peak"] <= 100


def test_manifest_scalar_column_runs_the_oracle():
    case = mf.Case("gemm_ex", "T", "N", mf.R16F, mf.R16F, mf.R32F, mf.F32, mf.Shape(300, 200, 100))
    ms, (m, n, k, batch) = bench._manifest_scalar_fn(case)
    assert (m, n, k, batch) == (128, 128, 100, 1) and ms > 0
    case = mf.Case("batched", "N", "N", mf.R32F, mf.R32F, mf.R32F, mf.F32, mf.Shape(512, 64, 512))
    ms, (m, n, k, batch) = bench._manifest_scalar_fn(case)
    assert (m, n, k, batch) == (256, 64, 256, 1)
    case = mf.Case("gemm_strided_batched_ex", "N", "N", mf.R8I, mf.R8I, mf.R32I, mf.I32, mf.Shape(64, 64, 64))
    assert bench._manifest_scalar_fn(case)[1] == (64, 64, 64, 2)


def _run(*args, timeout=300):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, env=env, cwd=ROOT)


def test_cli_without_gpu_manifest_mode_reports_invalid():
    p = _run("--manifest=all", "--sizes=128", "--no-cpu-baseline")
    assert p.returncode == 0
    assert json.loads(p.stdout.strip().splitlines()[-1]) == {"status": "invalid", "error": "no CUDA device available"}


def test_cli_reference_arm_prints_one_json_line():
    p = _run("--impl", "reference", "--steps", "3", "--warmup", "3", "--ref-seconds", "1.5")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = p.stdout.strip().splitlines()
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["unit"] == "TFLOP/s"


def test_cli_rejects_short_warmup():
    p = _run("--warmup", "2")
    assert p.returncode != 0


@pytest.mark.parametrize("units,parts,align", [(8192, 2, 256), (8192, 8, 256), (65536, 8, 256), (256, 8, 1),
                                               (64, 8, 1), (512, 4, 1), (1000, 3, 256), (100, 8, 256)])
def test_reference_arm_rank0_share_matches_the_library_plan(units, parts, align):
    import gemm_sm100 as gs

    assert bench.rank0_units(units, parts, align) == gs.plan_shards(units, parts, align)[1]


@pytest.mark.parametrize("name", ["c3-f16-nn", "c4-f16-strided", "c5b-i8-strided"])
@pytest.mark.parametrize("world,scaling", [(1, "weak"), (2, "weak"), (8, "strong")])
def test_both_arms_print_the_same_config_object(name, world, scaling):
    cfg0 = dict(bench.CONFIGS[name], name=name)
    ours, _ = bench.rank_share(cfg0, 0, world, scaling)
    theirs = dict(cfg0)
    key, align = ("batch", 1) if cfg0["shard"] == "batch" else ("n", 256)
    theirs[key] = bench.rank0_units(cfg0[key] * (world if scaling == "weak" else 1), world, align)
    assert bench.config_dict(cfg0, ours, world, scaling) == bench.config_dict(cfg0, theirs, world, scaling)


def test_roofline_carries_both_denominators():
    for name in ("c3-f16-nn", "c5-i8-nn", "c4-f16-strided"):
        cfg = bench.CONFIGS[name]
        flops, byts = bench.work(cfg)
        r = bench.roofline_of(cfg, flops, byts, 1.0, PEAKS, 123)
        assert r["peak_datasheet"] in (2250.0, 4500.0, 7700.0)
        assert abs(r["frac_datasheet"] - r["achieved"] / r["peak_datasheet"]) < 1e-3
        assert "not measured in this run" in r["traffic_source"]


def test_reference_arm_line_describes_one_whole_step():
    p = _run("--impl", "reference", "--config", "c5b-i8-strided", "--steps", "3", "--warmup", "3",
             "--ref-seconds", "1.5")
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads(p.stdout.strip().splitlines()[-1])
    assert 0 < d["sample_fraction"] < 1
    # ms_per_step is the whole configuration's step: the sample time scaled by 1 / sample_fraction
    assert d["ms_per_step"] == pytest.approx(d["ms_per_sample"] / d["sample_fraction"], rel=1e-2)
    assert d["config"]["name"] == "c5b-i8-strided" and d["config"]["per_rank"]["batch"] == 64


def test_cli_rejects_unknown_config_in_a_list():
    p = _run("--config", "c3-f16-nn,nope")
    assert p.returncode != 0 and "nope" in p.stderr


def test_tile_sweep_shape_lists_match_the_rule():
    """The shapes `bench.py --tile-sweep` times: well-formed, and every split-K shape is one the library splits
    (at least 4 slices), so the split-K profile measures the split path."""
    import gemm_sm100 as gs

    for shapes in (bench.TILE_SWEEP_SHAPES, bench.SPLITK_SHAPES):
        assert shapes and all(len(s) == 4 and all(isinstance(v, int) and v > 0 for v in s) for s in shapes)
    for m, n, k, b in bench.SPLITK_SHAPES:
        for at, ct, comp in ((gs.R_16F, gs.R_32F, gs.COMPUTE_32F), (gs.R_16BF, gs.R_16BF, gs.COMPUTE_32F)):
            st, tile, parts = gs.plan_tile(0, 0, m, n, k, at, ct, comp, batch=b)
            assert st == gs.STATUS_SUCCESS and parts >= 4, (m, n, k, parts)


def test_reference_arm_under_torchrun_world_two_prints_once():
    """The driver launches the reference arm like our own arm for N > 1 (torchrun, one process per GPU):
    rank 0 alone runs the sample and prints the line, with rank 0's share in `config`; rank 1 exits 0."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3", "--ref-seconds", "1.5"]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    # weak scaling: two ranks' worth of columns, rank 0 holding the first 8192 of 16384
    assert d["config"]["per_rank"]["n"] == 8192
