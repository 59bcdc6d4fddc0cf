"""Compat-call trace records in the reference's trace format.

The reference's compat bench writes one JSON object per line for every CUDA / cuBLAS call it
makes (reasons cudaMalloc, cudaMemcpyH2D, cublasSgemm, cudaMemcpyD2H, cudaFree): a `call`
record before, a `return` record after, a `retired_tile` record for each
GEMM tile retired in between (observed from the telemetry's tile counter) and one `final`
record (reference src/compat_bench/main.cpp:105-200, src/compat_bench/report.cpp:390-410,
schemas/cuda-compat-trace-v1.schema.json). `TracedCompat` produces the same records around
`xvram_b200.compat.CompatApi`, so tools that read the reference's traces read these.

Record fields (all required): schema_version 1, report_type "xvram.cuda_compat_trace",
sequence (from 1), monotonic_timestamp_ns (since the tracer started), operation_id,
allocation_id (integer or null), transition ("call" | "return" | "retired_tile" |
"final"), bytes, tiles_retired (cumulative), reason.
"""
from __future__ import annotations

import json
import time
from typing import IO, Optional

TRANSITIONS = ("call", "return", "retired_tile", "final")

BENCH_DIGEST_INIT = (1469598103934665603, 1099511628211 ^ 0x9E3779B97F4A7C15)
COMPAT_DIGEST_INIT = (1469598103934665603, 0x9E3779B97F4A7C15)


def _hex(state) -> str:
    return f"{state[1]:016x}{state[0]:016x}"


def bench_digest(data, absolute_offset: int = 0) -> str:
    """The reference GEMM bench's 128-bit digest of a byte buffer (numpy array or bytes)
    whose first byte sits at `absolute_offset` (xvram_b200_digest_bench)."""
    import ctypes as C

    import numpy as np

    from ._native import lib
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, bytes)
                               else data)
    state = (C.c_uint64 * 2)(*BENCH_DIGEST_INIT)
    lib.xvram_b200_digest_bench(buf.ctypes.data, buf.nbytes, absolute_offset, state)
    return _hex(state)


def compat_digest(values) -> str:
    """The reference compat bench's digest of FP32 values (xvram_b200_digest_compat)."""
    import ctypes as C

    import numpy as np

    from ._native import lib
    v = np.ascontiguousarray(values, dtype=np.float32)
    state = (C.c_uint64 * 2)(*COMPAT_DIGEST_INIT)
    lib.xvram_b200_digest_compat(v.ctypes.data, v.size, state)
    return _hex(state)


def trace_record(sequence: int, timestamp_ns: int, transition: str, operation_id: int,
                 allocation_id: Optional[int], nbytes: int, tiles_retired: int,
                 reason: str) -> dict:
    if transition not in TRANSITIONS:
        raise ValueError(f"unknown transition {transition!r}")
    if sequence < 1 or timestamp_ns < 0 or operation_id < 0 or nbytes < 0 or tiles_retired < 0:
        raise ValueError("trace counters are non-negative and sequence starts at 1")
    return {"schema_version": 1, "report_type": "xvram.cuda_compat_trace",
            "sequence": sequence, "monotonic_timestamp_ns": timestamp_ns,
            "operation_id": operation_id, "allocation_id": allocation_id,
            "transition": transition, "bytes": nbytes, "tiles_retired": tiles_retired,
            "reason": reason}


class TracedCompat:
    """Wraps a CompatApi: every malloc / free / memcpy / sgemm writes call and return
    records (and the tiles retired in between) to `sink`, one JSON object per line.
    Allocations are identified by sequence numbers given at malloc (as the reference's
    bench does), never by their addresses; a call on an interior pointer names the
    allocation that contains it."""

    def __init__(self, api, sink: IO[str]):
        self.api, self.sink = api, sink
        self.t0 = time.monotonic_ns()
        self.sequence = 0
        self.operation = 0
        self.tiles = int(api.telemetry().tiles_retired)
        self.records = 0
        self.next_allocation = 0
        self.allocations: dict[int, tuple[int, int]] = {}  # base -> (id, bytes)

    def _allocation(self, ptr: int):
        for base, (ident, size) in self.allocations.items():
            if base <= ptr < base + max(size, 1):
                return ident
        return None

    def _emit(self, transition, allocation, nbytes, reason):
        self.sequence += 1
        rec = trace_record(self.sequence, time.monotonic_ns() - self.t0, transition,
                           self.operation if transition != "final" else 0, allocation, nbytes,
                           self.tiles, reason)
        self.sink.write(json.dumps(rec, separators=(",", ":")) + "\n")
        self.records += 1

    def _retired(self):
        now = int(self.api.telemetry().tiles_retired)
        while self.tiles < now:
            self.tiles += 1
            self._emit("retired_tile", None, 0, "observed_event_retirement")

    def _traced(self, name, allocation, nbytes, fn):
        """A call record, the call, the tiles it retired, its return record.  A call that
        raises gets no return record (the reference's bench stops at its first failure),
        so the final record then closes the trace with that call still open."""
        self.operation += 1
        self._emit("call", allocation, nbytes, name)
        try:
            out = fn()
        finally:
            self._retired()
        self._emit("return", allocation, nbytes, name)
        return out

    # Reasons and fields as the reference's bench writes them for the CUDA / cuBLAS calls
    # these compat entries stand in for (src/compat_bench/executor.cpp:241-347).
    def malloc(self, nbytes):
        self.next_allocation += 1
        ident = self.next_allocation
        ptr = self._traced("cudaMalloc", ident, nbytes, lambda: self.api.malloc(nbytes))
        self.allocations[ptr] = (ident, nbytes)
        return ptr

    def free(self, ptr):
        ident = self._allocation(ptr)
        size = self.allocations.get(ptr, (None, 0))[1]
        out = self._traced("cudaFree", ident, size, lambda: self.api.free(ptr))
        self.allocations.pop(ptr, None)
        return out

    def h2d(self, dst, src_ptr, nbytes):
        return self._traced("cudaMemcpyH2D", self._allocation(dst), nbytes,
                            lambda: self.api.h2d(dst, src_ptr, nbytes))

    def d2h(self, dst_ptr, src, nbytes):
        return self._traced("cudaMemcpyD2H", self._allocation(src), nbytes,
                            lambda: self.api.d2h(dst_ptr, src, nbytes))

    def sgemm(self, h, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc):
        """No allocation id; bytes = the logical operand bytes 4 (mk + kn + mn)."""
        return self._traced("cublasSgemm", None, 4 * (m * k + k * n + m * n),
                            lambda: self.api.sgemm(h, op_a, op_b, m, n, k, alpha, a, lda, b,
                                                   ldb, beta, c, ldc))

    def close(self, ok: bool = True) -> None:
        self._retired()
        self._emit("final", None, 0, "completed" if ok else "failed")
        self.sink.flush()
