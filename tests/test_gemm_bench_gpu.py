"""The GEMM bench report on the B200: out-of-core runs (FP32 strict, FP32 through AUTO =
three-term TF32, FP16 with FP16 C, FP64) whose analytic results match bit for bit, with
the report's proof and cleanup claims all true."""
from __future__ import annotations

import json

import pytest

from xvram_b200 import gemm_bench

pytestmark = pytest.mark.gpu
MiB = 1 << 20


@pytest.mark.parametrize("dtype,c_dtype,compute", [("fp32", None, "fp32_strict"),
                                                   ("fp32", None, "auto"),
                                                   ("fp16", "fp16", "auto"),
                                                   ("fp64", None, "auto")])
def test_out_of_core_report(dtype, c_dtype, compute):
    # operands above the 32 MiB budget in every case (40-48 MiB before workspace)
    m, n, k = {"fp32": (2048, 2048, 2048), "fp16": (4096, 2048, 2048),
               "fp64": (2048, 1024, 1024)}[dtype]
    rep = gemm_bench.run(m, n, k, 0, 1, dtype, c_dtype, compute, 1.0, 1.0, passes=2,
                         cache_target_bytes=32 * MiB, chunk_bytes=2 * MiB)
    assert rep["outcome"]["status"] == "completed", rep["outcome"]
    assert rep["numerics"]["all_results_match"]
    assert rep["plans"][0]["tile_count"] > 1
    assert all(v is True for key, v in rep["proof"].items() if key.endswith("_verified"))
    assert rep["cache"]["resident_bytes_peak"] <= 32 * MiB
    assert all(rep["cleanup"].values())
    assert rep["device"]["compute_capability_major"] == 10
    json.dumps(rep)
