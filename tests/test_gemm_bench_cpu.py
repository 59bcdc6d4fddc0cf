"""The GEMM bench report (xvram.gemm_bench v1, xvram_b200/gemm_bench.py) on the host-memory
fake device: the analytic pattern against the oracle's restatement of the reference's
closed form (src/gemm_bench/pattern.cpp:215-237), out-of-core runs in FP32, FP16 and FP64
whose results match bit for bit, and the report checked against the reference's own
schema (schemas/gemm-bench-report-v1.schema.json, read when the reference tree is
present).  One field is known to differ: build.cuda_headers_version is this build's CUDA
12.9 (12090), while the schema asks for >= 13000, the reference's own toolkit."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from fake_device import installed
from oracle_lib import load_oracle
from schema_check import check

from xvram_b200 import gemm_bench

MiB = 1 << 20
from reference_tree import reference_dir

SCHEMA = reference_dir() / "schemas" / "gemm-bench-report-v1.schema.json"


def test_pattern_closed_form_matches_the_oracle():
    orc = load_oracle()
    rows = np.array([0, 1, 2, 3, 4, 10, 99], dtype=np.int64)
    cols = np.array([0, 1, 4, 5, 13], dtype=np.int64)
    for k in (1, 2, 3, 5, 6, 7, 64, 4096, 131072):
        got = gemm_bench.pattern_expected(rows[:, None], cols[None, :], k)
        for i, r in enumerate(rows):
            for j, c in enumerate(cols):
                assert int(got[i, j]) == orc.lib.xo_gb_expected(int(r), int(c), k)
                if k <= 64:  # and the closed form is the sum it stands for
                    p = np.arange(k)
                    direct = int(np.sum(gemm_bench.pattern_a(r, p) * gemm_bench.pattern_b(p, c)))
                    assert int(got[i, j]) == direct
    assert orc.lib.xo_gb_a(7, 3) == int(gemm_bench.pattern_a(np.int64(7), np.int64(3)))
    assert orc.lib.xo_gb_b(3, 7) == int(gemm_bench.pattern_b(np.int64(3), np.int64(7)))


def schema_violations(report):
    schema = json.loads(SCHEMA.read_text())
    errs = check(report, schema)
    known = [e for e in errs if e[0] == "$.build.cuda_headers_version" and "minimum 13000" in e[1]]
    return [e for e in errs if e not in known], known


CASES = [  # dtype, c_dtype, compute, op_a, op_b, alpha, beta, (m, n, k)
    ("fp32", None, "fp32_strict", 1, 0, 2.0, 1.0, (1536, 1280, 1024)),
    ("fp16", "fp16", "auto", 0, 1, 1.0, 0.0, (2048, 1536, 1536)),
    ("fp64", None, "auto", 0, 0, 1.0, -1.0, (1024, 768, 768)),
]


@pytest.mark.parametrize("dtype,c_dtype,compute,op_a,op_b,alpha,beta,shape", CASES)
def test_out_of_core_report_on_the_fake(dtype, c_dtype, compute, op_a, op_b, alpha, beta, shape):
    m, n, k = shape
    with installed():
        rep = gemm_bench.run(m, n, k, op_a, op_b, dtype, c_dtype, compute, alpha, beta,
                             passes=2, cache_target_bytes=16 * MiB, chunk_bytes=2 * MiB)
    assert rep["outcome"]["status"] == "completed" and rep["outcome"]["exit_code"] == 0
    assert rep["numerics"]["all_results_match"] and rep["numerics"]["mismatch_count"] == 0
    assert rep["numerics"]["elements_verified"] == m * n
    assert rep["plans"][0]["tile_count"] > 1
    assert rep["workloads"][0]["passes_completed"] == 2
    assert rep["workloads"][0]["tiles_retired"] == rep["workloads"][0]["tiles_total"]
    assert all(v is True for key, v in rep["proof"].items() if key.endswith("_verified"))
    assert rep["cache"]["resident_bytes_peak"] <= 16 * MiB
    assert all(rep["cleanup"].values())
    json.dumps(rep)  # serialisable as it stands
    if SCHEMA.exists():
        bad, known = schema_violations(rep)
        assert not bad, bad
        assert len(known) == 1


def test_schema_checker_sees_violations():
    """The checker itself: a report with a wrong enum, a missing field, an extra field and a
    broken conditional is rejected."""
    if not SCHEMA.exists():
        pytest.skip("reference schema not present")
    with installed():
        rep = gemm_bench.run(256, 256, 64, passes=1, compute="fp32_strict")
    rep["numerics"]["validation_mode"] = "eyeball"
    del rep["cache"]["mapping_count"]
    rep["plans"][0]["extra"] = 1
    rep["proof"]["all_workloads_match_reference"] = False  # completed reports must claim it
    bad, _ = schema_violations(rep)
    paths = {p for p, _ in bad}
    assert "$.numerics.validation_mode" in paths and "$.cache" in paths
    assert "$.plans[0]" in paths and "$.proof.all_workloads_match_reference" in paths


def test_inexact_scalars_are_refused():
    with pytest.raises(ValueError):
        gemm_bench.run(64, 64, 64, alpha=0.5)
