"""The compat bench (xvram_b200/compat_bench.py, report type xvram.cuda_compat v1) on the
host-memory fake device, in a child process (the compat table initialises once per
process): the suite scenario -- four padded smoke shapes in every operation pair, an
out-of-core GEMM through a 16 MiB budget, the rejection set -- completes with every proof
and cleanup claim true, its report passes the reference's schema
(schemas/cuda-compat-v1.schema.json, read when the reference tree is present), and its
trace is in the reference's trace format.  The pattern, the FP64 reference and the
padding layout are checked against the reference's own generator (golden fills) and
the oracle's restatement of its reference_result."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from fake_device import ROOT
from schema_check import check

from xvram_b200 import compat_bench

from reference_tree import reference_dir

SCHEMA = reference_dir() / "schemas" / "cuda-compat-v1.schema.json"
TRACE_SCHEMA = reference_dir() / "schemas" / "cuda-compat-trace-v1.schema.json"

SCRIPT = r"""
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from fake_device import installed
from xvram_b200 import compat_bench
with installed():
    rep = compat_bench.run(sys.argv[2], 1536, 1280, 1024, 0, 1, 3, 7, 0, 1.0, 1.0, 2,
                           16 << 20, 2 << 20, 0, sys.argv[3])
print(json.dumps(rep))
"""


def run_child(scenario: str, trace: Path) -> dict:
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), scenario, str(trace)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_fill_matches_the_reference_generator(golden):
    """The padded operand storage for the reference's 37 x 19 x 67 shape (padding 5,
    offset 11) equals the reference's fill_pattern output, bit for bit, for A, B and C in
    every operation pair (tests/golden/reference_vectors.json)."""
    g = golden["cb_padded_fills"]
    shp = g["shape"]
    for f in g["fills"]:
        want = np.frombuffer(bytes.fromhex(f["bits"]), np.float32)
        got = compat_bench.fill(shp["m"], shp["n"], shp["k"], f["ta"], f["tb"], shp["padding"],
                                shp["offset"], g["seed"], "abc"[f["operand"]])
        assert got.size == f["count"] and np.array_equal(got.view(np.uint32),
                                                          want.view(np.uint32)), f


def test_reference_matches_the_oracle():
    """The bench's FP64 reference (full and period-4 forms) against the oracle's
    restatement of the reference's reference_result."""
    from oracle_lib import load_oracle
    orc = load_oracle()
    m, n = 37, 19
    for k, full in ((67, True), (67, False), (4096, False), (1, True)):
        for seed, alpha, beta, passes in ((0, 1.0, 0.0, 1), (5, 0.5, -1.25, 2), (300, 2.0, 1.0, 3)):
            ref = compat_bench.reference(m, n, k, seed, alpha, beta, passes, full)
            for i, j in ((0, 0), (3, 7), (36, 18)):
                want = orc.lib.xo_cb_reference_result(i, j, k, seed, alpha, beta, passes,
                                                      1 if full else 0)
                assert abs(ref[j, i] - want) <= 1e-9 * max(1.0, abs(want)), (k, full, i, j)


def test_suite_on_the_fake(tmp_path):
    trace = tmp_path / "trace.jsonl"
    rep = run_child("suite", trace)
    assert rep["outcome"] == {"status": "completed", "exit_code": 0, "reason": "proof_completed",
                              "message": rep["outcome"]["message"]}
    assert [w["name"] for w in rep["workloads"]] == ["smoke_nn", "smoke_nt", "smoke_tn",
                                                     "smoke_tt", "gemm"]
    assert all(w["mismatches"] == 0 and w["digest"] == w["reference_digest"] or
               w["reference_kind"] == "cpu_fp64_analytic_periodic_v1" for w in rep["workloads"])
    assert rep["compatibility"]["rejections_checked"] == 8
    assert rep["compatibility"]["rejections_failed"] == 0
    assert all(rep["proof"].values()) and all(rep["cleanup"].values())
    gemm = rep["workloads"][-1]
    assert gemm["logical_bytes"] > 16 << 20 and gemm["handle_reuses"] > 0
    if SCHEMA.exists():
        assert check(rep, json.loads(SCHEMA.read_text())) == []
    lines = [json.loads(x) for x in trace.read_text().splitlines()]
    assert lines[-1]["transition"] == "final" and lines[-1]["reason"] == "completed"
    assert [r["sequence"] for r in lines] == list(range(1, len(lines) + 1))
    assert rep["execution"]["trace_records"] == len(lines)
    if TRACE_SCHEMA.exists():
        ts = json.loads(TRACE_SCHEMA.read_text())
        assert all(check(r, ts) == [] for r in lines)


def test_rejection_scenario_on_the_fake(tmp_path):
    rep = run_child("rejection", tmp_path / "t.jsonl")
    assert rep["workloads"] == [] and rep["compatibility"]["rejections_failed"] == 0
    # no GEMM workload: nothing oversubscribed, so the proof is incomplete by design
    assert rep["outcome"]["exit_code"] == 27
    assert rep["proof"]["real_oversubscription_reuse"] is False
    if SCHEMA.exists():
        assert check(rep, json.loads(SCHEMA.read_text())) == []
