"""The reference CLI's JSONL rows for this backend on a B200 (bench.py's manifest mode, the counterpart of
bench/gemm_perf.zig:91-158): every timed row validates the library's C against cuBLAS's on the same
buffers, so a run at a tiny size must produce rows with no `validation_failed` status, at least one
hardware-accelerated `ok` row, and the summary line (bench/gemm_perf.zig:76-88)."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_manifest_rows_validate_on_the_gpu(cuda, tmp_path):
    out = tmp_path / "rows.jsonl"
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--manifest=all", "--sizes=128", "--iters=2",
                        "--warmup=3", "--only-cublas-supported", "--no-cpu-baseline", f"--output={out}"], capture_output=True, text=True, timeout=900,
                       cwd=ROOT)
    assert p.returncode == 0, p.stderr[-3000:]
    rows = [json.loads(x) for x in open(out) if x.strip()]
    statuses = [r.get("status") for r in rows if "status" in r]
    assert statuses, "no rows"
    assert "validation_failed" not in statuses, [r for r in rows if r.get("status") == "validation_failed"][:3]
    assert statuses.count("ok") + statuses.count("perf_regression") > 0
    summary = [r for r in rows if r.get("summary") == "hardware_accelerated"]
    assert len(summary) == 1 and summary[0]["cases"] > 0
