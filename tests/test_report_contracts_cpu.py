"""The bench reports and traces, judged by the reference's own contract scripts.

* tests/contract/gemm_contract.py: its completed-report semantics (tiles retired = tiles
  planned, the logical data larger than the device, the working set inside the cache
  target, mappings = access grants = unmaps, dirty evictions = write-backs, no unsafe
  remaps, output digest = expected digest, no raw addresses) applied to this library's
  out-of-core GEMM bench report on the host-memory fake device, whose total memory is set
  below the operands.
* tests/contract/compat_contract.py: schema, semantics (one post-shutdown snapshot: every
  frame unmapped and handle released, transactions = tiles retired, event boundaries =
  unmaps, calls attempted = completed + rejected, host ledger within the host store cap)
  and the trace rules (one public call at a time, tiles retired only inside a cublasSgemm
  call, a final record) for the compat bench's "gemm" scenario on the fake device; and the
  same script on a suite report plus trace that the compat bench wrote on a B200
  (tests/golden/compat_suite_b200.json, made by tests/golden/make_compat_suite_b200.sh),
  where the reference's ordinary-cuBLAS baseline ran too.

The scripts are read in place from the reference tree; every test skips without it.
"""
from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import pytest

from fake_device import ROOT, installed
from reference_tree import reference_dir, reference_file
from schema_check import check

MiB = 1 << 20
GOLDEN = Path(__file__).resolve().parent / "golden"


def _contract(name: str) -> Path:
    p = reference_file("tests", "contract", name)
    if p is None:
        pytest.skip("reference tree not present")
    pytest.importorskip("jsonschema")
    return p


def _run_compat_contract(report: Path, trace: Path) -> subprocess.CompletedProcess:
    script = _contract("compat_contract.py")
    schemas = reference_dir() / "schemas"
    return subprocess.run(
        [sys.executable, str(script), "--schema", str(schemas / "cuda-compat-v1.schema.json"),
         "--trace-schema", str(schemas / "cuda-compat-trace-v1.schema.json"),
         "--report", str(report), "--trace", str(trace)],
        cwd=script.parent, capture_output=True, text=True, timeout=300)


def test_gemm_bench_report_meets_the_reference_gemm_contract():
    script = _contract("gemm_contract.py")
    spec = importlib.util.spec_from_file_location("reference_gemm_contract", script)
    contract = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(contract)
    from xvram_b200 import gemm_bench
    # 48 MiB of operands on a device that reports 32 MiB in total, through a 16 MiB cache
    with installed(free_bytes=1 << 30, total_bytes=32 * MiB):
        rep = gemm_bench.run(2048, 2048, 2048, 1, 0, "fp32", None, "fp32_strict", 2.0, 1.0,
                             passes=1, cache_target_bytes=16 * MiB, chunk_bytes=2 * MiB)
    assert rep["outcome"]["exit_code"] == 0
    contract.assert_completed_semantics(rep)
    schema = json.loads((reference_dir() / "schemas" /
                         "gemm-bench-report-v1.schema.json").read_text())
    # the one known difference: this build's CUDA headers are 12.9, the schema asks >= 13.0
    assert [e for e in check(rep, schema) if e[0] != "$.build.cuda_headers_version"] == []


CHILD = r"""
import json, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
from fake_device import installed
from xvram_b200 import compat_bench
with installed():
    rep = compat_bench.run("gemm", 1536, 1280, 1024, 0, 1, 3, 7, 0, 1.0, 1.0, 2,
                           16 << 20, 2 << 20, 0, sys.argv[3])
open(sys.argv[2], "w").write(json.dumps(rep))
"""


def test_compat_gemm_report_and_trace_meet_the_reference_compat_contract(tmp_path):
    _contract("compat_contract.py")
    report, trace = tmp_path / "compat.json", tmp_path / "trace.jsonl"
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(report), str(trace)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    rep = json.loads(report.read_text())
    assert rep["outcome"]["exit_code"] == 0, rep["outcome"]
    out = _run_compat_contract(report, trace)
    assert out.returncode == 0 and "contracts passed" in out.stdout, out.stdout + out.stderr


def test_b200_suite_report_meets_the_reference_compat_contract():
    report, trace = GOLDEN / "compat_suite_b200.json", GOLDEN / "compat_suite_b200_trace.jsonl"
    _contract("compat_contract.py")
    if not report.exists():
        pytest.skip("no B200 report committed")
    rep = json.loads(report.read_text())
    small = [w for w in rep["workloads"] if w["reference_kind"] == "cpu_fp64_full"]
    assert len(small) == 4 and all(w["native_baseline_equal"] is True for w in small)
    out = _run_compat_contract(report, trace)
    assert out.returncode == 0 and "contracts passed" in out.stdout, out.stdout + out.stderr
