"""Compat-table bench with the reference's report format (report_type xvram.cuda_compat,
schema version 1; reference schemas/cuda-compat-v1.schema.json, executor
src/compat_bench/executor.cpp:180-420, operands src/compat_bench/pattern.cpp).

    python -m xvram_b200.compat_bench --scenario suite --m 4096 --n 4096 --k 4096 \\
        --cache-target-mib 128 --chunk-mib 2 --report compat.json [--trace trace.jsonl]

Drives this library's xvram_cuda_compat_get_api table the way a CUDA / cuBLAS program
does: cudaMalloc-style allocations, cudaMemcpy of the operands, cublasSgemm `passes`
times, cudaMemcpy of C back, cudaFree.  Operands are the reference compat bench's
patterns, stored with `padding` extra rows per column and `offset` elements before and
after the matrix, all filled with the padding value:

    a(i, p) = (1 + (i + seed % 3) % 3) * {1, -1, 0.5, 0.5}[p % 4]
    b(p, j) = (1 + (j + (seed >> 8) % 3) % 3) * {1, 1, 0.5, 0.5}[p % 4]
    c(i, j) = (1 + (i + j) % 7) / 4,     padding -1234.5

Scenarios, as in the reference: "suite" runs four small shapes (37 x 19 x 67, padding 5,
offset 11, every operation pair), the requested "gemm" shape and the rejection checks;
"gemm" runs the requested shape; "rejection" runs only the rejection checks.  Every C
element is checked: a matrix element against an FP64 reference of `passes` updates
C = alpha A B + beta C (a full FP64 sum for small shapes, the pattern's period-4 closed
form for large ones) within 1e-4 + 2e-5 |ref|, a padding element bit for bit.  Each
rejection check makes an unsupported call and requires it to fail without submitting
work (tiles, mappings and copied bytes unchanged).  Digests are the reference compat
bench's.  For the small shapes the reference's ordinary-cuBLAS baseline runs too
(native_baseline_*: the same storage through cublasGemmEx in pedantic FP32, every stored
element within the tolerance of this library's); on a host without a CUDA device (the
fake device) those fields are null.

The compat table allows one initialisation per process: run this as its own process.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import platform
import subprocess
import time
from pathlib import Path

import numpy as np

from . import compat as cp
from .gemm_bench import timing
from .report import TracedCompat, compat_digest

# The report's cache section: the adapter session's runtime telemetry, field for field.
CACHE_FIELDS = (
    "cache_target_bytes", "cache_target_minimum_bytes", "cache_target_maximum_bytes",
    "resident_bytes", "resident_bytes_peak", "workspace_bytes", "bytes_h2d", "bytes_d2h",
    "cache_hits", "cache_misses", "clean_evictions", "dirty_evictions", "writebacks_completed",
    "mappings", "unmaps", "set_access_calls", "handle_reuses", "unsafe_remaps",
    "unsafe_transitions", "budget_shrinks", "budget_grows", "physical_handles_created",
    "physical_handles_released", "event_boundaries", "pinned_staging_bytes",
    "transactions_completed", "algorithm_selections", "algorithm_cache_hits",
    "budget_sample_count", "cuda_free_bytes_minimum", "cuda_free_bytes_end",
    "wddm_available_bytes_minimum", "wddm_available_bytes_end", "wddm_budget_observed",
    "watchdog_rejections", "target_oom_retries", "last_transaction_ms")

PADDING_VALUE = np.float32(-1234.5)
_A_SIGN = np.array([1.0, -1.0, 0.5, 0.5], dtype=np.float32)
_B_SIGN = np.array([1.0, 1.0, 0.5, 0.5], dtype=np.float32)
MAX_ABS, MAX_REL = 1e-4, 2e-5
OP_T, OP_N, OP_C = 1, 0, 2


# ------------------------------------------------------------------ the reference pattern
def pattern_a(i, p, seed):
    return (1 + (i + seed % 3) % 3).astype(np.float32) * _A_SIGN[p % 4]


def pattern_b(p, j, seed):
    return (1 + (j + (seed >> 8) % 3) % 3).astype(np.float32) * _B_SIGN[p % 4]


def pattern_c(i, j):
    return (1 + (i + j) % 7).astype(np.float32) * np.float32(0.25)


def storage(m, n, k, op_a, op_b, padding, offset, operand):
    """(rows, columns, ld, elements) of one operand's storage: ld = rows + padding, and
    `offset` padding elements before the matrix and after it."""
    if operand == "a":
        rows, cols = (k, m) if op_a else (m, k)
    elif operand == "b":
        rows, cols = (n, k) if op_b else (k, n)
    else:
        rows, cols = m, n
    ld = rows + padding
    return rows, cols, ld, ld * cols + 2 * offset


def fill(m, n, k, op_a, op_b, padding, offset, seed, operand) -> np.ndarray:
    rows, cols, ld, elements = storage(m, n, k, op_a, op_b, padding, offset, operand)
    out = np.full(elements, PADDING_VALUE, dtype=np.float32)
    r = np.arange(rows, dtype=np.int64)[None, :]
    c = np.arange(cols, dtype=np.int64)[:, None]
    if operand == "a":
        vals = pattern_a(c, r, seed) if op_a else pattern_a(r, c, seed)
    elif operand == "b":
        vals = pattern_b(c, r, seed) if op_b else pattern_b(r, c, seed)
    else:
        vals = pattern_c(r, c)
    body = out[offset:offset + ld * cols].reshape(cols, ld)
    body[:, :rows] = vals
    return out


def reference(m, n, k, seed, alpha, beta, passes, full) -> np.ndarray:
    """(n, m) FP64 result of `passes` updates C = alpha op(A) op(B) + beta C from c(i, j)."""
    i = np.arange(m, dtype=np.int64)[None, :]
    j = np.arange(n, dtype=np.int64)[:, None]
    if full:
        p = np.arange(k, dtype=np.int64)
        A = pattern_a(np.arange(m, dtype=np.int64)[:, None], p[None, :], seed).astype(np.float64)
        B = pattern_b(p[:, None], np.arange(n, dtype=np.int64)[None, :], seed).astype(np.float64)
        dot = (A @ B).T  # (n, m)
    else:  # a period of 4 in p sums to 0.5 * a(i, 0) b(0, j); the rest added directly
        scale = pattern_a(i, np.int64(0), seed).astype(np.float64) * \
            pattern_b(np.int64(0), j, seed).astype(np.float64)
        dot = (k // 4) * 0.5 * scale
        for p in range(k % 4):
            dot = dot + pattern_a(i, np.int64(p), seed).astype(np.float64) * \
                pattern_b(np.int64(p), j, seed).astype(np.float64)
    result = pattern_c(i, j).astype(np.float64)
    for _ in range(passes):
        result = float(np.float32(alpha)) * dot + float(np.float32(beta)) * result
    return result


def close_enough(actual: np.ndarray, expected: np.ndarray) -> np.ndarray:
    return np.isfinite(actual) & np.isfinite(expected) & \
        (np.abs(actual - expected) <= MAX_ABS + MAX_REL * np.abs(expected))


# ------------------------------------------------------------------ the run
def run(scenario="suite", m=4096, n=4096, k=4096, op_a=0, op_b=0, padding=0, offset=0, seed=0,
        alpha=1.0, beta=0.0, passes=1, cache_target_bytes=0, chunk_bytes=64 << 20,
        device=0, trace_path=None) -> dict:
    generated = datetime.datetime.now(datetime.timezone.utc).isoformat().replace("+00:00", "Z")
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.device_ordinal = device
    cfg.session.cache_target_bytes = cache_target_bytes
    cfg.session.chunk_size_bytes = chunk_bytes
    sink = open(trace_path, "w") if trace_path else None
    diagnostics: list[str] = []
    workloads: list[dict] = []
    rejections_checked = rejections_failed = 0
    exit_code, reason, message = 27, "execution_failure", ""
    tel_first = tel_last = None
    initialized = False
    calls = None
    try:
        st = api.initialize(cfg)
        if st != cp.SUCCESS:
            raise cp.XvramError("initialize", st, api.error())
        initialized = True
        tel_first = api.telemetry()
        calls = TracedCompat(api, sink) if sink else api
        h = api.blas_create()
        api.check("blas_set_math_mode", api.t.blas_set_math_mode(h, 2))      # pedantic
        api.check("blas_set_pointer_mode", api.t.blas_set_pointer_mode(h, 0))  # host
        api.check("blas_set_stream", api.t.blas_set_stream(h, 0))
        shapes = []
        if scenario == "suite":
            for a in (0, 1):
                for b in (0, 1):
                    shapes.append((f"smoke_{'nt'[a]}{'nt'[b]}", 37, 19, 67, 5, 11, a, b))
        if scenario != "rejection":
            shapes.append(("gemm", m, n, k, padding, offset, op_a, op_b))
        for name, sm, sn, sk, pad, off, sa, sb in shapes:
            workloads.append(run_workload(api, calls, h, name, sm, sn, sk, pad, off, sa, sb,
                                          seed, alpha, beta, passes, device))
            if workloads[-1]["mismatches"]:
                raise RuntimeError("CPU reference or padding verification failed")
        if scenario in ("suite", "rejection"):
            rejections_checked, rejections_failed = run_rejections(api, h, device, alpha, beta)
            if rejections_failed:
                exit_code, reason = 27, "execution_failure"
                raise RuntimeError("unsupported call was not rejected before submission")
        api.synchronize()
        api.blas_destroy(h)
        exit_code, reason = 0, "proof_completed"
        message = "selected synchronous CUDA/cuBLAS compatibility proof completed"
    except Exception as e:  # the report records the failure
        if exit_code == 27 and workloads and workloads[-1]["mismatches"]:
            exit_code, reason = 24, "reference_mismatch"
        message = str(e) or type(e).__name__
        diagnostics.append(message)
    finally:
        if initialized:
            tel_last = api.telemetry()
        closed = api.shutdown() == cp.SUCCESS if initialized else False
        tel_closed = None
        if initialized:
            out = cp.CompatTelemetry()
            out.struct_size = C.sizeof(cp.CompatTelemetry)
            if api.t.get_telemetry(C.byref(out)) == cp.SUCCESS:
                tel_closed = out
        trace_records = 0
        if sink:
            if isinstance(calls, TracedCompat):
                calls.close(ok=exit_code == 0)
                trace_records = calls.records
            sink.close()
    return build_report(generated, scenario, m, n, k, op_a, op_b, padding, offset, seed, alpha,
                        beta, passes, cfg, device, workloads, rejections_checked,
                        rejections_failed, tel_first, tel_last, tel_closed, closed,
                        exit_code, reason, message, diagnostics, bool(sink), trace_records)


def native_baseline(arrays, lds, m, n, k, offset, op_a, op_b, alpha, beta, passes, device):
    """The reference's native baseline (src/compat_bench/native_baseline.cpp:10-130): the
    same padded operand storage copied to the device and `passes` ordinary cuBLAS calls
    (cublasGemmEx, CUBLAS_COMPUTE_32F_PEDANTIC, pedantic math; xvram_b200.native_baseline),
    each followed by a stream synchronisation, timed together on the host clock.  Returns
    C's storage and those milliseconds, or None on a host without a CUDA device (the
    host-memory fake device), where the report's native_baseline_* fields stay null.  Like
    the reference it takes small resident cases only (each operand at most 16 MiB)."""
    try:
        import torch
    except ImportError:
        return None
    if not torch.cuda.is_available():
        return None
    from .native_baseline import PedanticSgemm
    if any(a.nbytes > 16 << 20 for a in arrays):
        raise RuntimeError("baseline is limited to small resident cases")
    dev = torch.device("cuda", device)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.device(dev), torch.cuda.stream(stream):
        t = [torch.from_numpy(a).to(dev) for a in arrays]
        stream.synchronize()
        with PedanticSgemm(stream.cuda_stream) as gemm:
            t0 = time.perf_counter()
            for _ in range(passes):
                gemm(op_a, op_b, m, n, k, alpha, t[0].data_ptr() + 4 * offset, lds[0],
                     t[1].data_ptr() + 4 * offset, lds[1], beta, t[2].data_ptr() + 4 * offset,
                     lds[2])
                stream.synchronize()
            ms = (time.perf_counter() - t0) * 1e3
        c = t[2].cpu().numpy()
    return c, ms


def run_workload(api, calls, h, name, m, n, k, padding, offset, op_a, op_b, seed, alpha, beta,
                 passes, device=0) -> dict:
    before = api.telemetry()
    arrays = [fill(m, n, k, op_a, op_b, padding, offset, seed, w) for w in "abc"]
    lds = [storage(m, n, k, op_a, op_b, padding, offset, w)[2] for w in "abc"]
    ptrs = []
    for arr in arrays:
        p = calls.malloc(arr.nbytes)
        ptrs.append(p)
        calls.h2d(p, arr.ctypes.data, arr.nbytes)
    timings = []
    for _ in range(passes):
        t0 = time.perf_counter()
        st = calls.sgemm(h, op_a, op_b, m, n, k, alpha, ptrs[0] + 4 * offset, lds[0],
                         ptrs[1] + 4 * offset, lds[1], beta, ptrs[2] + 4 * offset, lds[2])
        api.check("blas_sgemm", st)
        timings.append((time.perf_counter() - t0) * 1e3)
    out = np.empty_like(arrays[2])
    calls.d2h(out.ctypes.data, ptrs[2], out.nbytes)
    full = m <= 128 and n <= 128 and k <= 512
    ref = reference(m, n, k, seed, alpha, beta, passes, full)
    ld = lds[2]
    body = out[offset:offset + ld * n].reshape(n, ld)
    actual = body[:, :m].astype(np.float64)
    ok = close_enough(actual, ref)
    expected = np.full_like(out, PADDING_VALUE)
    expected[offset:offset + ld * n].reshape(n, ld)[:, :m] = ref.astype(np.float32)
    material = np.zeros(out.size, dtype=bool)
    material[offset:offset + ld * n].reshape(n, ld)[:, :m] = True
    pad_ok = out.view(np.uint32)[~material] == np.float32(PADDING_VALUE).view(np.uint32)
    bad = np.zeros(out.size, dtype=bool)
    bad[material] = ~ok.reshape(-1)
    bad[~material] = ~pad_ok
    native_equal = native_ms = None
    if full:
        # every stored element, matrix and padding, against the ordinary cuBLAS result
        # (reference src/compat_bench/executor.cpp:278-284, 326-329)
        baseline = native_baseline(arrays, lds, m, n, k, offset, op_a, op_b, alpha, beta,
                                   passes, device)
        if baseline is not None:
            base_ok = close_enough(out.astype(np.float64), baseline[0].astype(np.float64))
            bad |= ~base_ok
            native_equal, native_ms = bool(base_ok.all()), float(baseline[1])
    err = np.abs(actual - ref)
    for p in ptrs:
        calls.free(p)
    after = api.telemetry()
    d = lambda f: int(getattr(after.runtime, f) - getattr(before.runtime, f))
    return {
        "name": name, "status": "completed" if not bad.any() else "corruption",
        "m": m, "n": n, "k": k, "padding_elements": padding, "offset_elements": offset,
        "logical_bytes": 4 * (m * k + k * n + m * n),
        "storage_bytes": int(sum(a.nbytes for a in arrays)),
        "passes_completed": passes,
        "output_elements_checked": int(m * n),
        "padding_elements_checked": int((~material).sum()),
        "mismatches": int(bad.sum()),
        "tiles_retired": int(after.tiles_retired - before.tiles_retired),
        "mappings": d("mappings"), "unmaps": d("unmaps"),
        "h2d_bytes": d("bytes_h2d"), "d2h_bytes": d("bytes_d2h"),
        "evictions": d("clean_evictions") + d("dirty_evictions"),
        "handle_reuses": d("handle_reuses"),
        "op_a": "nt"[op_a], "op_b": "nt"[op_b],
        "mismatch_offset": int(np.argmax(bad)) * 4 if bad.any() else None,
        "max_absolute_error": float(err.max()) if err.size else 0.0,
        "max_relative_error": float((err / np.maximum(np.abs(ref), 1e-30)).max()) if err.size
        else 0.0,
        "digest": compat_digest(out), "reference_digest": compat_digest(expected),
        "reference_kind": "cpu_fp64_full" if full else "cpu_fp64_analytic_periodic_v1",
        "native_baseline_equal": native_equal, "native_baseline_ms": native_ms,
        "pass_timings": timing(timings),
    }


def run_rejections(api, h, device, alpha, beta) -> tuple[int, int]:
    """The reference's rejection set (executor.cpp:364-404): each call must fail without
    submitting tiles, mapping frames or copying bytes."""
    foreign = np.ones(1, dtype=np.float32)
    fp = foreign.ctypes.data
    al, be = C.c_float(alpha), C.c_float(beta)
    checks = [
        lambda: api.t.set_device(device + 1) != cp.SUCCESS,
        lambda: api.t.blas_set_pointer_mode(h, 1) != cp.SUCCESS,          # device pointers
        lambda: api.t.blas_set_stream(h, 1) != cp.SUCCESS,                # a foreign stream
        lambda: api.t.free_device(fp) != cp.SUCCESS,                      # not ours
        lambda: api.t.memcpy(fp, fp, 4, 3) != cp.SUCCESS,                 # device to device
        lambda: api.t.memcpy(fp, fp, 4, 4) != cp.SUCCESS,                 # default kind
        lambda: api.t.blas_sgemm(h, OP_N, OP_N, 0, 1, 1, C.byref(al), fp, 1, fp, 1,
                                 C.byref(be), fp, 1) != cp.SUCCESS,       # m = 0
        lambda: api.t.blas_sgemm(h, OP_C, OP_N, 1, 1, 1, C.byref(al), fp, 1, fp, 1,
                                 C.byref(be), fp, 1) != cp.SUCCESS,       # conjugate transpose
    ]
    failed = 0
    for call in checks:
        before = api.telemetry()
        rejected = call()
        after = api.telemetry()
        if (not rejected or after.tiles_submitted != before.tiles_submitted or
                after.runtime.mappings != before.runtime.mappings or
                after.runtime.bytes_h2d != before.runtime.bytes_h2d or
                after.runtime.bytes_d2h != before.runtime.bytes_d2h):
            failed += 1
    return len(checks), failed


def _git_commit() -> str:
    try:
        r = subprocess.run(["git", "rev-parse", "HEAD"], cwd=Path(__file__).resolve().parent,
                           capture_output=True, text=True, timeout=10)
        return r.stdout.strip() or "unknown"
    except (OSError, subprocess.SubprocessError):
        return "unknown"


def build_report(generated, scenario, m, n, k, op_a, op_b, padding, offset, seed, alpha, beta,
                 passes, cfg, device, workloads, rejections_checked, rejections_failed,
                 tel_first, tel_last, tel_closed, closed, exit_code, reason, message,
                 diagnostics, trace_enabled, trace_records) -> dict:
    from .gemm_bench import device_query
    dev = device_query(device)
    # One snapshot for the whole report, taken after shutdown, as the reference's executor
    # does (src/compat_bench/executor.cpp:433-447): the cache counters then show every
    # frame unmapped and every physical handle released.
    fin = tel_closed or tel_last or tel_first
    last = fin
    rt = last.runtime if last is not None else None
    u = lambda x: int(x) if x is not None else 0
    mismatches = sum(w["mismatches"] for w in workloads)
    gemm = [w for w in workloads if w["name"] == "gemm"]
    cache_target = u(rt.cache_target_maximum_bytes) if rt else 0
    cleanup = {
        "operations_drained": bool(closed and fin and fin.cleanup_operations_drained),
        "events_drained": bool(closed and fin and fin.cleanup_events_drained),
        "allocations_released": bool(fin and fin.allocations_released == fin.allocations_created),
        "handles_destroyed": bool(fin and fin.handles_destroyed == fin.handles_created),
        "reservations_freed": bool(fin and fin.retired_va_reservations == 0 and
                                   fin.retired_va_bytes == 0),
        "adapter_closed": bool(closed), "worker_terminated": bool(closed),
        "trace_closed": True,
    }
    proof = None if rt is None else {
        # every call was either completed through the adapter or one of the rejections
        # checked here (attempted == completed + rejected at quiescence)
        "supported_calls_routed": bool(last.calls_attempted == last.calls_completed +
                                       last.calls_rejected and
                                       last.calls_rejected == rejections_checked and
                                       last.calls_completed > 0),
        "reference_equal": bool(workloads) and mismatches == 0,
        "padding_preserved": all(w["mismatches"] == 0 for w in workloads),
        "rejections_before_submission": rejections_failed == 0,
        "stable_addresses": bool(rt.flags & 1),
        "no_physical_aliases": bool(rt.flags & 2) and rt.unsafe_remaps == 0,
        "mapping_access_balanced": rt.set_access_calls == rt.mappings,
        "mapping_unmap_balanced": bool(fin and fin.runtime.unmaps == fin.runtime.mappings),
        "event_safe": rt.unsafe_transitions == 0,
        "zero_unsafe_activity": rt.unsafe_remaps == 0 and rt.unsafe_transitions == 0,
        "bounded_cache": rt.resident_bytes_peak <= rt.cache_target_maximum_bytes,
        "real_oversubscription_reuse": bool(gemm) and gemm[0]["logical_bytes"] > cache_target
        and gemm[0]["handle_reuses"] > 0,
        "cleanup_complete": all(cleanup.values()),
    }
    if exit_code == 0 and proof and not all(proof.values()):
        exit_code, reason = 27, "execution_failure"
        message = "proof incomplete: " + ", ".join(k for k, v in proof.items() if not v)
        diagnostics.append(message)
    status = "completed" if exit_code == 0 else ("corruption" if exit_code == 24 else
                                                 "oom" if exit_code == 25 else "failed")
    total_mem = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    return {
        "schema_version": 1,
        "report_type": "xvram.cuda_compat",
        "generated_at_utc": generated,
        "build": {"version": "xvram_b200 0.1", "git_commit": _git_commit(),
                  "build_type": "Release",
                  "cuda_headers_version": int(dev.runtime_headers_version) if dev else 0},
        "system": {"os_name": platform.system() or "unknown", "os_version": platform.release(),
                   "architecture": platform.machine() or "unknown",
                   "logical_processor_count": os.cpu_count() or 0,
                   "physical_memory_bytes": total_mem,
                   "available_memory_bytes": u(last.host_available_bytes) if last else 0},
        "device": {"ordinal": device,
                   "name": (last.device_name.decode(errors="replace") if last else "") or "unknown",
                   "total_memory_bytes": u(last.total_vram_bytes) if last else 0,
                   "cuda_driver_version": u(rt.cuda_driver_version) if rt else 0,
                   "cublas_version": 0, "cublas_lt_version": 0, "cublas_library_source": 0,
                   "uuid": None, "pci_bus_id": None},
        "configuration": {
            "scenario": scenario, "policy": "lru",
            "requested_logical_bytes": 4 * (m * k + k * n + m * n) if scenario != "rejection"
            else None,
            "requested_m": m if scenario != "rejection" else None,
            "requested_n": n if scenario != "rejection" else None,
            "requested_k": k if scenario != "rejection" else None,
            "chunk_bytes": int(cfg.session.chunk_size_bytes),
            "cache_target_bytes": int(cfg.session.cache_target_bytes),
            "device_headroom_bytes": int(cfg.session.device_headroom_bytes),
            "workspace_bytes": int(cfg.session.workspace_cap_bytes),
            "staging_slots": int(cfg.session.staging_slots),
            "prefetch_distance": int(cfg.session.prefetch_distance),
            "budget_poll_ms": int(cfg.session.budget_poll_ms),
            "stall_timeout_ms": int(cfg.stall_timeout_ms), "timeout_ms": 600000,
            "passes": passes, "padding_elements": padding, "offset_elements": offset,
            "seed": seed, "alpha": float(alpha), "beta": float(beta),
            "op_a": "nt"[op_a], "op_b": "nt"[op_b], "trace_enabled": trace_enabled,
            "identifiers_included": False, "compression": "disabled",
            "effective_chunk_bytes": u(last.effective_chunk_bytes) if last else 0,
            "host_store_cap_bytes": u(last.host_store_cap_bytes) if last else 0,
            "host_headroom_bytes": u(last.host_headroom_bytes) if last else 0,
            "host_budget_bytes": u(last.host_budget_bytes) if last else 0,
        },
        "compatibility": {
            "abi_version": 1, "profile": "synchronous_fp32_sgemm", "native_fallback": False,
            "calls_submitted": u(last.calls_submitted) if last else 0,
            "calls_completed": u(last.calls_completed) if last else 0,
            "calls_rejected": u(last.calls_rejected) if last else 0,
            "rejections_checked": rejections_checked, "rejections_failed": rejections_failed,
            "allocations_created": u(fin.allocations_created) if fin else 0,
            "allocations_released": u(fin.allocations_released) if fin else 0,
            "live_allocations": u(fin.live_allocations) if fin else 0,
            "handles_created": u(fin.handles_created) if fin else 0,
            "handles_destroyed": u(fin.handles_destroyed) if fin else 0,
            "live_handles": u(fin.live_handles) if fin else 0,
            "retired_va_reservations": u(fin.retired_va_reservations) if fin else 0,
            "retired_va_reservations_freed": u(fin.retired_va_reservations_freed) if fin else 0,
            "calls_attempted": u(last.calls_attempted) if last else 0,
            "retired_va_bytes": u(fin.retired_va_bytes) if fin else 0,
            "retired_va_bytes_freed": u(fin.retired_va_bytes_freed) if fin else 0,
        },
        "workloads": workloads,
        "execution": {
            "telemetry_observed": last is not None,
            "gemm_calls": u(last.gemm_calls) if last else 0,
            "tiles_submitted": u(last.tiles_submitted) if last else 0,
            "tiles_retired": u(last.tiles_retired) if last else 0,
            "progress_sequence": u(last.progress_sequence) if last else 0,
            "host_h2d_bytes": u(last.h2d_bytes) if last else 0,
            "host_d2h_bytes": u(last.d2h_bytes) if last else 0,
            "logical_bytes_peak": u(last.logical_bytes_peak) if last else 0,
            "host_backing_peak_bytes": u(last.host_backing_peak_bytes) if last else 0,
            "trace_records": trace_records, "trace_complete": trace_enabled,
        },
        "cache": None if rt is None else {
            f: (float(getattr(rt, f)) if f == "last_transaction_ms" else int(getattr(rt, f)))
            for f in CACHE_FIELDS},
        "verification": {
            "absolute_tolerance": MAX_ABS, "relative_tolerance": MAX_REL,
            "mismatches": mismatches,
            "output_elements_checked": sum(w["output_elements_checked"] for w in workloads),
            "max_absolute_error": max((w["max_absolute_error"] for w in workloads), default=0.0),
        },
        "proof": proof,
        "outcome": {"status": status, "exit_code": exit_code, "reason": reason,
                    "message": message},
        "cleanup": cleanup,
        "diagnostics": diagnostics,
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--scenario", choices=["suite", "gemm", "rejection"], default="suite")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--op-a", choices=["n", "t"], default="n")
    ap.add_argument("--op-b", choices=["n", "t"], default="n")
    ap.add_argument("--padding", type=int, default=0)
    ap.add_argument("--offset", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--alpha", type=float, default=1.0)
    ap.add_argument("--beta", type=float, default=0.0)
    ap.add_argument("--passes", type=int, default=1)
    ap.add_argument("--cache-target-mib", type=int, default=0)
    ap.add_argument("--chunk-mib", type=int, default=64)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--report", default=None)
    ap.add_argument("--trace", default=None, help="xvram.cuda_compat_trace JSON lines")
    a = ap.parse_args()
    rep = run(a.scenario, a.m, a.n, a.k, int(a.op_a == "t"), int(a.op_b == "t"), a.padding,
              a.offset, a.seed, a.alpha, a.beta, a.passes, a.cache_target_mib << 20,
              a.chunk_mib << 20, a.device, a.trace)
    if a.report:
        Path(a.report).write_text(json.dumps(rep, indent=1) + "\n")
    print(json.dumps({"status": rep["outcome"]["status"], "exit_code": rep["outcome"]["exit_code"],
                      "reason": rep["outcome"]["reason"],
                      "workloads": [(w["name"], w["mismatches"]) for w in rep["workloads"]],
                      "rejections": (rep["compatibility"]["rejections_checked"],
                                     rep["compatibility"]["rejections_failed"])}))
    raise SystemExit(rep["outcome"]["exit_code"])


if __name__ == "__main__":
    main()
