"""Compat trace records (xvram_b200.report) against the reference's trace format
(reference schemas/cuda-compat-trace-v1.schema.json, restated here as checks) and the
call / return / retired_tile / final sequence its compat bench writes
(reference src/compat_bench/main.cpp:105-200)."""
from __future__ import annotations

import io
import json

import pytest

from xvram_b200.report import TracedCompat, trace_record

REQUIRED = ["schema_version", "report_type", "sequence", "monotonic_timestamp_ns",
            "operation_id", "allocation_id", "transition", "bytes", "tiles_retired", "reason"]


def check_schema(rec: dict) -> None:
    assert sorted(rec) == sorted(REQUIRED)          # required, no additional properties
    assert rec["schema_version"] == 1
    assert rec["report_type"] == "xvram.cuda_compat_trace"
    for key in ("sequence", "monotonic_timestamp_ns", "operation_id", "bytes", "tiles_retired"):
        assert isinstance(rec[key], int) and not isinstance(rec[key], bool) and rec[key] >= 0
    assert rec["sequence"] >= 1
    assert rec["allocation_id"] is None or (isinstance(rec["allocation_id"], int) and
                                            rec["allocation_id"] >= 0)
    assert rec["transition"] in ("call", "return", "retired_tile", "final")
    assert isinstance(rec["reason"], str)


def test_record_fields_and_limits():
    check_schema(trace_record(1, 0, "call", 1, 4096, 64, 0, "cudaMalloc"))
    check_schema(trace_record(2, 5, "final", 0, None, 0, 3, "completed"))
    with pytest.raises(ValueError):
        trace_record(0, 0, "call", 1, None, 0, 0, "x")
    with pytest.raises(ValueError):
        trace_record(1, 0, "begin", 1, None, 0, 0, "x")


class FakeCompat:
    """Host-only stand-in for the compat table: counts calls, retires two tiles per sgemm."""

    class Tel:
        def __init__(self, tiles):
            self.tiles_retired = tiles

    def __init__(self):
        self.tiles = 0

    def telemetry(self):
        return self.Tel(self.tiles)

    def malloc(self, n):
        return 0x1000

    def free(self, p):
        return None

    def h2d(self, dst, src, n):
        return None

    def d2h(self, dst, src, n):
        return None

    def sgemm(self, *args):
        self.tiles += 2
        return 0


def test_traced_call_sequence():
    sink = io.StringIO()
    tr = TracedCompat(FakeCompat(), sink)
    p = tr.malloc(256)
    tr.h2d(p, 0, 256)
    assert tr.sgemm(1, 0, 0, 8, 8, 8, 1.0, p, 8, p, 8, 0.0, p, 8) == 0
    tr.d2h(0, p, 256)
    tr.free(p)
    tr.close()
    recs = [json.loads(line) for line in sink.getvalue().splitlines()]
    for r in recs:
        check_schema(r)
    assert [r["sequence"] for r in recs] == list(range(1, len(recs) + 1))
    kinds = [r["transition"] for r in recs]
    assert kinds[-1] == "final" and kinds.count("final") == 1
    assert kinds.count("call") == kinds.count("return") == 5
    assert kinds.count("retired_tile") == 2
    gemm_call = next(r for r in recs if r["reason"] == "cublasSgemm" and r["transition"] == "call")
    assert gemm_call["allocation_id"] is None and gemm_call["bytes"] == 4 * 3 * 64
    assert [r["reason"] for r in recs if r["transition"] == "call"] == [
        "cudaMalloc", "cudaMemcpyH2D", "cublasSgemm", "cudaMemcpyD2H", "cudaFree"]
    tiles = [r for r in recs if r["transition"] == "retired_tile"]
    assert all(t["operation_id"] == gemm_call["operation_id"] for t in tiles)
    assert [t["tiles_retired"] for t in tiles] == [1, 2]
    times = [r["monotonic_timestamp_ns"] for r in recs]
    assert times == sorted(times)


def test_compat_digest_matches_the_reference_implementation(ref_lib):
    """The compat bench digest against the reference's own Digest (compiled in oracle/_ref)."""
    import ctypes as C

    import numpy as np

    from xvram_b200.report import compat_digest
    if not hasattr(ref_lib, "xr_cb_digest"):
        import pytest
        pytest.skip("reference shim predates xr_cb_digest")
    ref_lib.xr_cb_digest.argtypes = [C.c_void_p, C.c_uint64, C.c_char_p]
    rng = np.random.default_rng(3)
    for count in (0, 1, 7, 1000):
        v = rng.uniform(-1e3, 1e3, count).astype(np.float32)
        out = C.create_string_buffer(33)
        ref_lib.xr_cb_digest(v.ctypes.data, count, out)
        assert compat_digest(v) == out.value.decode()


def test_bench_digest_follows_its_definition():
    """The GEMM bench digest (reference src/gemm_bench/executor.cpp:42-65) against a plain
    restatement of its two lanes, including a non-zero starting offset."""
    import numpy as np

    from xvram_b200.report import BENCH_DIGEST_INIT, bench_digest
    mask = (1 << 64) - 1

    def slow(data: bytes, offset: int) -> str:
        low, high = BENCH_DIGEST_INIT
        for i, v in enumerate(data):
            idx = offset + i
            low = ((low ^ (v + (idx & 0xFF))) * 1099511628211) & mask
            high = ((high ^ (v + 0x9E + (idx >> 8))) * 0x100000001B3) & mask
            high ^= high >> 29
        return f"{high:016x}{low:016x}"
    data = np.random.default_rng(5).integers(0, 256, 3000, dtype=np.uint8)
    for off in (0, 1, 255, 70000):
        assert bench_digest(data, off) == slow(data.tobytes(), off)
