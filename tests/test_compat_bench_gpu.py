"""The compat bench on the B200 (child process: one compat initialisation per process):
the suite scenario with an out-of-core GEMM through a 64 MiB budget completes with every
proof and cleanup claim true; the four small shapes also match the reference's
ordinary-cuBLAS baseline (cublasGemmEx, pedantic FP32) element for element within the
bench's tolerance; the post-shutdown counters reconcile as the reference's compat
contract asks."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_suite_on_the_gpu(tmp_path):
    report = tmp_path / "compat.json"
    r = subprocess.run([sys.executable, "-m", "xvram_b200.compat_bench", "--scenario", "suite",
                        "--m", "4096", "--n", "3072", "--k", "2048", "--padding", "3",
                        "--offset", "5", "--passes", "2", "--beta", "1", "--cache-target-mib",
                        "64", "--chunk-mib", "2", "--report", str(report), "--trace",
                        str(tmp_path / "trace.jsonl")],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    rep = json.loads(report.read_text())
    assert rep["outcome"]["status"] == "completed"
    assert all(w["mismatches"] == 0 for w in rep["workloads"])
    assert all(rep["proof"].values()) and all(rep["cleanup"].values())
    assert rep["compatibility"]["rejections_failed"] == 0
    small = [w for w in rep["workloads"] if w["reference_kind"] == "cpu_fp64_full"]
    assert len(small) == 4
    assert all(w["native_baseline_equal"] is True and w["native_baseline_ms"] > 0
               for w in small)
    cache, execution = rep["cache"], rep["execution"]
    assert cache["transactions_completed"] == execution["tiles_retired"]
    assert cache["mappings"] == cache["set_access_calls"] == cache["unmaps"]
    assert cache["event_boundaries"] == cache["unmaps"] and cache["resident_bytes"] == 0
    assert cache["physical_handles_created"] == cache["physical_handles_released"]
    assert rep["compatibility"]["retired_va_reservations"] == 0
    assert execution["host_backing_peak_bytes"] <= rep["configuration"]["host_store_cap_bytes"]
