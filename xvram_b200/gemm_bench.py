"""Out-of-core GEMM bench with the reference's report format (report_type xvram.gemm_bench,
schema version 1; reference schemas/gemm-bench-report-v1.schema.json, writer
src/gemm_bench/report_json.cpp, executor src/gemm_bench/executor.cpp).

    python -m xvram_b200.gemm_bench --m 4096 --n 4096 --k 4096 --cache-target-mib 64 \\
        --chunk-mib 2 --dtype fp32 --passes 2 --report gemm_bench.json

One GEMM plan runs through the SDK (xvram_get_api) on a session whose device budget is
--cache-target-mib, `passes` times.  The operands carry the reference bench's analytic
integer pattern (src/gemm_bench/pattern.cpp:215-237):

    a(i, p) = 1 + i % 3 + p % 2,   b(p, j) = 1 + j % 5 + p % 3,
    sum_p a(i, p) b(p, j) in closed form,

whose products and sums are small integers, exact in every element type and arithmetic
the bench runs, so validation is "structured" against an "analytic" reference: every
output element is compared bit for bit with the closed form rounded once to C's type.
With beta != 0, C starts as c(i, j) = 1 + (i + j) % 4 and is rewritten before every pass.
alpha and beta must be integers of magnitude at most 16 (the result stays exact).

The report fills every field of the schema from this run: plans and workloads from
gemm_plan_get_info and the operations' info, cache and telemetry from the session's
telemetry, proof from checks made here (see `proof`).  Differences from the reference's
writer, all stated in the report's own terms:
  * digests are the reference bench's 128-bit digest of C's bytes (column-major, from
    byte offset 0), expected and actual;
  * build.cuda_headers_version is the CUDA runtime version the library was built with
    (12090 here); the reference's schema asks for >= 13000 because the reference itself
    needs CUDA 13;
  * cuBLAS fields are null / false: no cuBLAS is used;
  * tile, H2D, D2H and write-back timings have no samples (the executor times whole
    operations), the GEMM timing has one sample per pass.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import platform
import statistics
import subprocess
import time
from pathlib import Path

import numpy as np

from . import sdk
from ._native import DeviceInfo, lib
from .report import bench_digest

DTYPES = {"fp16": sdk.FP16, "bf16": sdk.BF16, "fp32": sdk.FP32, "fp64": sdk.FP64}
DTYPE_NAMES = {v: k for k, v in DTYPES.items()}
COMPUTE = {"auto": sdk.COMPUTE_AUTO, "fp32_strict": sdk.COMPUTE_FP32_STRICT,
           "tf32": sdk.COMPUTE_FP32_TF32, "fp64": sdk.COMPUTE_FP64}
COMPUTE_NAMES = {v: k for k, v in COMPUTE.items()}
ESIZE = {sdk.FP16: 2, sdk.BF16: 2, sdk.FP32: 4, sdk.FP64: 8}


# ------------------------------------------------------------------ analytic pattern
def pattern_a(rows: np.ndarray, p: np.ndarray) -> np.ndarray:
    return 1 + rows % 3 + p % 2


def pattern_b(p: np.ndarray, cols: np.ndarray) -> np.ndarray:
    return 1 + cols % 5 + p % 3


def pattern_expected(rows: np.ndarray, cols: np.ndarray, k: int) -> np.ndarray:
    """sum_{p < k} a(i, p) b(p, j), exactly (int64), for broadcastable rows / cols."""
    a = 1 + rows % 3
    b = 1 + cols % 5
    sum_p = k // 2                                   # sum of p % 2
    sum_q = 3 * (k // 3) + (1 if k % 3 == 2 else 0)  # sum of p % 3
    sum_pq = 3 * (k // 6) + (0, 0, 1, 1, 1, 1)[k % 6]  # sum of (p % 2)(p % 3)
    return k * a * b + a * sum_q + b * sum_p + sum_pq


def pattern_c(rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    return 1 + (rows + cols) % 4


def encode(values: np.ndarray, dtype: int) -> np.ndarray:
    """Exact-integer (or float64) values -> the stored array of `dtype`, rounded to
    nearest even (FP16 / BF16 as uint16 bit patterns)."""
    v = np.asarray(values, dtype=np.float64)
    if dtype == sdk.FP16:
        return v.astype(np.float16).view(np.uint16)
    if dtype == sdk.BF16:
        u = v.astype(np.float32).view(np.uint32).astype(np.uint64)
        u = u + 0x7FFF + ((u >> 16) & 1)
        return (u >> 16).astype(np.uint16)
    if dtype == sdk.FP32:
        return v.astype(np.float32)
    return v


def decode(stored: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == sdk.FP16:
        return stored.view(np.float16).astype(np.float64)
    if dtype == sdk.BF16:
        return (stored.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return stored.astype(np.float64)


def digest128(arr: np.ndarray) -> str:
    """The reference bench's digest of C's bytes (column-major, from offset 0)."""
    return bench_digest(np.ascontiguousarray(arr).view(np.uint8))


def stored_operand(which: str, op: int, m: int, n: int, k: int, dtype: int) -> np.ndarray:
    """Column-major storage (as a (columns, rows) array) of A (op(A) m x k) or B
    (op(B) k x n) for operation op (0 = N, 1 = T), tight leading dimension."""
    if which == "a":
        i = np.arange(m, dtype=np.int64)[:, None]
        p = np.arange(k, dtype=np.int64)[None, :]
        logical = pattern_a(i, p)                      # m x k
    else:
        p = np.arange(k, dtype=np.int64)[:, None]
        j = np.arange(n, dtype=np.int64)[None, :]
        logical = pattern_b(p, j)                      # k x n
    stored = logical if op == 0 else logical.T     # the stored rows x columns
    return encode(np.ascontiguousarray(stored.T), dtype)  # column-major: columns first


def timing(samples: list[float]) -> dict:
    if not samples:
        return {"sample_count": 0, "total_ms": None, "minimum_ms": None, "median_ms": None,
                "p95_ms": None, "maximum_ms": None}
    s = sorted(samples)
    return {"sample_count": len(s), "total_ms": float(sum(s)), "minimum_ms": float(s[0]),
            "median_ms": float(statistics.median(s)),
            "p95_ms": float(s[min(len(s) - 1, int(round(0.95 * (len(s) - 1))))]),
            "maximum_ms": float(s[-1])}


def device_query(ordinal: int) -> DeviceInfo | None:
    d = DeviceInfo(struct_size=C.sizeof(DeviceInfo))
    return d if lib.xvram_b200_device_query(ordinal, C.byref(d)) == 0 else None


def _git_commit() -> str:
    try:
        r = subprocess.run(["git", "rev-parse", "HEAD"], cwd=Path(__file__).resolve().parent,
                           capture_output=True, text=True, timeout=10)
        return r.stdout.strip() or "unknown"
    except (OSError, subprocess.SubprocessError):
        return "unknown"


def _memory() -> tuple[int | None, int | None]:
    total = avail = None
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            key, val = line.split(":", 1)
            if key == "MemTotal":
                total = int(val.split()[0]) * 1024
            elif key == "MemAvailable":
                avail = int(val.split()[0]) * 1024
    except OSError:
        pass
    return total, avail


# ------------------------------------------------------------------ the run
def run(m: int, n: int, k: int, op_a: int = 0, op_b: int = 0, dtype: str = "fp32",
        c_dtype: str | None = None, compute: str = "auto", alpha: float = 1.0,
        beta: float = 0.0, passes: int = 1, cache_target_bytes: int = 0,
        chunk_bytes: int = 64 << 20, device_ordinal: int = 0, budget_poll_ms: int = 100,
        workspace_cap_bytes: int = 4 << 20) -> dict:
    """Runs the bench and returns the report (a dict in the xvram.gemm_bench v1 format)."""
    if alpha != int(alpha) or beta != int(beta) or abs(alpha) > 16 or abs(beta) > 16:
        raise ValueError("alpha and beta must be integers of magnitude <= 16 "
                         "(the analytic reference must stay exact)")
    ab = DTYPES[dtype]
    ct = DTYPES[c_dtype] if c_dtype else (sdk.FP64 if ab == sdk.FP64 else
                                          ab if ab in (sdk.FP16, sdk.BF16) else sdk.FP32)
    started = time.perf_counter()
    generated = datetime.datetime.now(datetime.timezone.utc).isoformat().replace("+00:00", "Z")
    dev0 = device_query(device_ordinal)
    cfg = sdk.session_config(device_ordinal=device_ordinal, cache_target_bytes=cache_target_bytes,
                             chunk_size_bytes=chunk_bytes, budget_poll_ms=budget_poll_ms,
                             workspace_cap_bytes=workspace_cap_bytes)
    s = sdk.Sdk(cfg)
    closed_ok = False
    try:
        tel0 = s.telemetry()
        A = stored_operand("a", op_a, m, n, k, ab)
        B = stored_operand("b", op_b, m, n, k, ab)
        rows = np.arange(m, dtype=np.int64)[None, :]
        cols = np.arange(n, dtype=np.int64)[:, None]
        c0 = encode(pattern_c(rows, cols), ct) if beta != 0 else np.zeros((n, m),
                                                                           dtype=encode(0, ct).dtype)
        exact = alpha * pattern_expected(rows, cols, k) + (beta * pattern_c(rows, cols)
                                                           if beta != 0 else 0)
        expected = encode(exact, ct)
        allocs = []
        for arr in (A, B, c0):
            h = s.alloc(arr.nbytes)
            h.write(np.ascontiguousarray(arr))
            allocs.append(h)
        Ad, Bd, Cd = allocs
        lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
        desc = s.gemm_desc(
            sdk.matrix(Ad, m if op_a == 0 else k, k if op_a == 0 else m, lda, data_type=ab),
            sdk.matrix(Bd, k if op_b == 0 else n, n if op_b == 0 else k, ldb, data_type=ab),
            sdk.matrix(Cd, m, n, m, data_type=ct), op_a, op_b, alpha=float(alpha),
            beta=float(beta), mode=COMPUTE[compute])
        t0 = time.perf_counter()
        plan = s.plan(desc)
        plan_ms = (time.perf_counter() - t0) * 1e3
        info = s.plan_info(plan)
        gemm_ms, ops = [], []
        for p in range(passes):
            if p and beta != 0:
                Cd.write(c0)  # every pass computes the same result
            op = C.c_void_p()
            t0 = time.perf_counter()
            s.check("gemm_submit", s.t.gemm_submit(plan, C.byref(op)))
            oi = s.wait(op.value)
            gemm_ms.append((time.perf_counter() - t0) * 1e3)
            s.t.operation_release(op.value)
            if oi.state != sdk.COMPLETED:
                raise sdk.SdkError("gemm", oi.result, s.error())
            ops.append(oi)
        s.t.gemm_plan_release(plan)
        out = np.empty_like(expected)
        Cd.read(out)
        stable = all(a.info().stable_virtual_address == 1 for a in allocs)
        tel = s.telemetry()
        for a in allocs:
            a.release()
        closed_ok = s.t.session_close(s.session, sdk.TIMEOUT_INFINITE) == sdk.SUCCESS
        final = s.telemetry()  # the snapshot taken after the runtime closed
    finally:
        if s.session:
            s.t.session_release(s.session)
            s.session = C.c_void_p()
    dev1 = device_query(device_ordinal)
    total_ms = (time.perf_counter() - started) * 1e3

    # numerics: bit-for-bit against the closed form in C's type
    diff = out.reshape(-1) != expected.reshape(-1)
    mismatches = int(diff.sum())
    first = int(np.argmax(diff)) * ESIZE[ct] if mismatches else None
    err = np.abs(decode(out, ct) - decode(expected, ct))
    ref_mag = np.abs(decode(expected, ct))
    max_abs = float(err.max()) if err.size else 0.0
    max_rel = float((err / np.where(ref_mag > 0, ref_mag, 1.0)).max()) if err.size else 0.0
    exp_digest, out_digest = digest128(expected), digest128(out)
    all_match = mismatches == 0 and exp_digest == out_digest

    logical = int(A.nbytes + B.nbytes + expected.nbytes)
    target0 = int(tel0.cache_target_bytes)
    flop = 2.0 * m * n * k
    tiles = int(info.tile_count)
    work_bytes_h2d = int(sum(o.bytes_h2d for o in ops))
    work_bytes_d2h = int(sum(o.bytes_d2h for o in ops))
    hits, misses = int(sum(o.cache_hits for o in ops)), int(sum(o.cache_misses for o in ops))
    best = min(gemm_ms) if gemm_ms else None
    effective = COMPUTE_NAMES.get(int(info.effective_compute_mode), "auto")
    status = "completed" if all_match else "failed"

    def rate(h, mi):
        return (h / (h + mi)) if (h + mi) else None

    report = {
        "schema_version": 1,
        "report_type": "xvram.gemm_bench",
        "generated_at_utc": generated,
        "build": {
            "version": "xvram_b200 0.1",
            "git_commit": _git_commit(),
            "compiler": f"nvcc (CUDA runtime {dev0.runtime_headers_version if dev0 else 0}) "
                        "-gencode arch=compute_100a,code=sm_100a; g++",
            "build_type": "Release",
            "cuda_headers_version": int(dev0.runtime_headers_version) if dev0 else 0,
        },
        "system": {
            "os_name": platform.system() or "unknown",
            "os_version": platform.release(),
            "architecture": platform.machine() or "unknown",
            "logical_processor_count": os.cpu_count() or 0,
            "physical_memory_bytes": _memory()[0],
            "available_memory_bytes": _memory()[1],
        },
        "device": None if dev0 is None else {
            "ordinal": int(dev0.ordinal),
            "name": dev0.name.decode(errors="replace") or "unknown",
            "uuid": None, "luid": None, "pci_bus_id": None,
            "driver_model": None,
            "total_memory_bytes": int(dev0.total_bytes),
            "free_memory_bytes_start": int(dev0.free_bytes),
            "free_memory_bytes_end": int(dev1.free_bytes) if dev1 else None,
            "safe_device_budget_bytes": int(tel.cache_target_maximum_bytes),
            "wddm_budget_bytes_start": None, "wddm_usage_bytes_start": None,
            "wddm_available_bytes_start": None, "wddm_available_bytes_minimum": None,
            "wddm_available_bytes_end": None,
            "vmm_supported": True, "uva_supported": True,
            "minimum_granularity_bytes": int(dev0.vmm_granularity) or None,
            "recommended_granularity_bytes": int(dev0.vmm_granularity) or None,
            "compute_capability_major": int(dev0.compute_capability_major),
            "compute_capability_minor": int(dev0.compute_capability_minor),
        },
        "configuration": {
            "requested_device_ordinal": device_ordinal,
            "requested_m": m, "requested_n": n, "requested_k": k,
            "scenario": "oversubscribed" if logical > target0 else "resident",
            "a_data_type": DTYPE_NAMES[ab], "b_data_type": DTYPE_NAMES[ab],
            "c_data_type": DTYPE_NAMES[ct], "compute_mode": compute,
            "a_layout": "column_major", "b_layout": "column_major", "c_layout": "column_major",
            "a_operation": "nt"[op_a], "b_operation": "nt"[op_b],
            "alpha": float(alpha), "beta": float(beta),
            "requested_chunk_bytes": chunk_bytes, "effective_chunk_bytes": chunk_bytes,
            "requested_cache_target_bytes": cache_target_bytes or None,
            "initial_cache_target_bytes": target0 or None,
            "requested_workspace_cap_bytes": workspace_cap_bytes,
            "effective_workspace_cap_bytes": workspace_cap_bytes,
            "context_mode": "isolated", "policy": "lru",
            "staging_slots": int(cfg.staging_slots), "prefetch_distance": int(cfg.prefetch_distance),
            "passes": passes, "budget_poll_ms": budget_poll_ms,
            "stall_timeout_ms": 250, "timeout_ms": 600000, "max_tile_ms": 600000,
            "identifiers_included": False,
        },
        "plans": [{
            "plan_id": 1, "status": status, "m": m, "n": n, "k": k,
            "a_data_type": DTYPE_NAMES[ab], "b_data_type": DTYPE_NAMES[ab],
            "c_data_type": DTYPE_NAMES[ct], "effective_compute_mode": effective,
            "tile_m": int(info.tile_m), "tile_n": int(info.tile_n), "tile_k": int(info.tile_k),
            "tile_count": tiles, "maximum_working_set_bytes": int(info.maximum_working_set_bytes),
            "workspace_bytes": int(info.workspace_bytes), "uses_cublas_lt": False,
            "heuristic_algorithm_count": None, "replan_count": 0,
        }],
        "workloads": [{
            "name": f"gemm_{dtype}_{m}x{n}x{k}_{'nt'[op_a]}{'nt'[op_b]}",
            "plan_id": 1, "status": status, "passes_completed": len(ops),
            "tiles_total": tiles * passes, "tiles_retired": int(sum(o.units_completed for o in ops)),
            "logical_allocation_bytes": logical, "oversubscribed": logical > target0,
            "cache_hits": hits, "cache_misses": misses, "cache_hit_rate": rate(hits, misses),
            "bytes_h2d": work_bytes_h2d, "bytes_d2h": work_bytes_d2h,
            "clean_evictions": int(tel.clean_evictions), "dirty_evictions": int(tel.dirty_evictions),
            "writebacks_completed": int(tel.writebacks_completed),
            "mapping_count": int(tel.mappings), "unmap_count": int(tel.unmaps),
            "set_access_count": int(tel.set_access_calls),
            "handle_reuse_count": int(tel.handle_reuses),
            "event_boundary_count": int(tel.event_boundaries),
            "unsafe_remap_count": int(tel.unsafe_remaps),
            "unsafe_transition_count": int(tel.unsafe_transitions),
            "elapsed_ms": float(sum(gemm_ms)),
            "achieved_tflops": flop / (best * 1e-3) / 1e12 if best else None,
            "output_digest128": out_digest,
        }],
        "numerics": {
            "validation_mode": "structured", "reference_precision": "analytic",
            "absolute_tolerance": 0.0, "relative_tolerance": 0.0,
            "maximum_absolute_error": max_abs, "maximum_relative_error": max_rel,
            "elements_verified": int(out.size), "mismatch_count": mismatches,
            "first_mismatch_byte_offset": first,
            "expected_digest128": exp_digest, "output_digest128": out_digest,
            "all_results_match": all_match,
        },
        "cache": {
            "target_bytes_initial": target0,
            "target_bytes_minimum": int(tel.cache_target_minimum_bytes),
            "target_bytes_maximum": int(tel.cache_target_maximum_bytes),
            "target_bytes_end": int(tel.cache_target_bytes),
            "resident_bytes_peak": int(tel.resident_bytes_peak),
            "pinned_staging_bytes": int(tel.pinned_staging_bytes),
            "workspace_bytes_peak": int(info.workspace_bytes),
            "physical_frame_count_peak": -(-int(tel.resident_bytes_peak) // chunk_bytes),
            "physical_handle_create_count": int(final.physical_handles_created),
            "physical_handle_release_count": int(final.physical_handles_released),
            "handle_reuse_count": int(tel.handle_reuses),
            "mapping_count": int(tel.mappings), "unmap_count": int(tel.unmaps),
            "set_access_count": int(tel.set_access_calls),
            "event_boundary_count": int(tel.event_boundaries),
            "unsafe_remap_count": int(tel.unsafe_remaps),
            "unsafe_transition_count": int(tel.unsafe_transitions),
            "cache_hits": int(tel.cache_hits), "cache_misses": int(tel.cache_misses),
            "cache_hit_rate": rate(int(tel.cache_hits), int(tel.cache_misses)),
            "clean_evictions": int(tel.clean_evictions), "dirty_evictions": int(tel.dirty_evictions),
            "writebacks_completed": int(tel.writebacks_completed),
            "target_shrink_count": int(tel.budget_shrinks), "target_grow_count": int(tel.budget_grows),
            "target_oom_retry_count": int(tel.target_oom_retries),
        },
        "telemetry": {
            "cuda_driver_version": int(tel.cuda_driver_version),
            "cublas_version": None, "cublas_lt_version": None, "cublas_lt_available": False,
            "cublas_library_source": None,
            "algorithms_selected": int(tel.algorithm_selections),
            "algorithm_cache_hits": int(tel.algorithm_cache_hits),
            "budget_sample_count": int(tel.budget_sample_count),
            "cuda_free_bytes_minimum": int(tel.cuda_free_bytes_minimum),
            "cuda_free_bytes_end": int(tel.cuda_free_bytes_end),
            "wddm_available_bytes_minimum": None, "wddm_available_bytes_end": None,
            "replans": 0, "watchdog_rejections": int(tel.watchdog_rejections),
            "total_elapsed_ms": total_ms,
            "plan_timing": timing([plan_ms]), "tile_timing": timing([]),
            "gemm_timing": timing(gemm_ms), "h2d_timing": timing([]), "d2h_timing": timing([]),
            "writeback_timing": timing([]),
        },
        "proof": proof(tel, info, logical, dev0, stable, all_match, tiles, workspace_cap_bytes),
        "outcome": {
            "status": status, "reason": None if all_match else "result mismatch",
            "exit_code": 0 if all_match else 70, "stage": None if all_match else "validate",
            "operation": None if all_match else "compare", "native_code": None,
            "native_name": None,
            "message": None if all_match else f"{mismatches} elements differ",
            "plan_id": None if all_match else 1, "tile_sequence": None,
            "logical_byte_offset": first,
        },
        "cleanup": cleanup(closed_ok, final),
        "diagnostics": [],
    }
    return report


def cleanup(closed_ok: bool, final) -> dict:
    """Teardown evidence: session_close succeeded (it drains the queue, closes the runtime --
    streams, events, workspace, reservations -- and stops the worker), and the telemetry
    snapshot taken after the runtime closed shows every mapping removed, every physical
    handle released and no host backing left.  No cuBLAS handle is ever created."""
    maps_removed = int(final.unmaps) == int(final.mappings)
    handles = int(final.physical_handles_released) == int(final.physical_handles_created)
    backing = int(final.pinned_staging_bytes) == 0
    out = {"operations_drained": closed_ok, "events_drained": closed_ok,
           "events_destroyed": closed_ok, "streams_destroyed": closed_ok,
           "cublas_handles_destroyed": True, "mappings_removed": closed_ok and maps_removed,
           "physical_handles_released": closed_ok and handles,
           "workspace_released": closed_ok, "virtual_reservations_released": closed_ok,
           "pinned_staging_released": closed_ok and backing,
           "host_backing_released": closed_ok and backing, "context_released": closed_ok,
           "worker_terminated": closed_ok}
    return {"complete": all(out.values()), **out}


def proof(tel, info, logical: int, dev, stable: bool, all_match: bool, tiles: int,
          workspace_cap: int) -> dict:
    """The report's proof section, each claim from an observation of this run:
    tiled execution (more than one tile), handle reuse and mappings (telemetry counters),
    stable addresses (the runtime's invariant flag and every allocation's
    stable_virtual_address after the run), no aliases (the flag and zero unsafe remaps or
    transitions), a write-back of C, the device budget (resident peak <= maximum target),
    the kernel workspace within the budget, and the results."""
    flags = int(tel.flags)
    target_max = int(tel.cache_target_maximum_bytes)
    workspace = int(info.workspace_bytes)
    return {
        "logical_allocation_bytes": logical,
        "total_vram_bytes": int(dev.total_bytes) if dev else None,
        "maximum_cache_target_bytes": target_max,
        "maximum_working_set_bytes": int(info.maximum_working_set_bytes),
        # The kernels' workspace is carved from the frame budget, not a separate pool.
        "workspace_cap_bytes": target_max,
        "logical_data_exceeds_vram": bool(dev) and logical > int(dev.total_bytes),
        "cache_smaller_than_logical": target_max < logical,
        "tiled_execution_verified": tiles > 1,
        "handles_reused": int(tel.handle_reuses) > 0,
        "stable_virtual_addresses_verified": stable and bool(flags & 1),
        "set_access_after_map_verified": int(tel.set_access_calls) >= int(tel.mappings) > 0,
        "event_boundaries_verified": int(tel.event_boundaries) > 0,
        "no_physical_aliases_verified": bool(flags & 2) and int(tel.unsafe_remaps) == 0 and
                                        int(tel.unsafe_transitions) == 0,
        "dirty_writeback_verified": int(tel.writebacks_completed) > 0 and all_match,
        "cache_target_respected": int(tel.resident_bytes_peak) <= target_max,
        "workspace_bounded": workspace <= target_max,
        "all_workloads_match_reference": all_match,
        "raw_virtual_addresses_omitted": True,
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--op-a", choices=["n", "t"], default="n")
    ap.add_argument("--op-b", choices=["n", "t"], default="n")
    ap.add_argument("--dtype", choices=list(DTYPES), default="fp32")
    ap.add_argument("--c-dtype", choices=list(DTYPES), default=None)
    ap.add_argument("--compute", choices=list(COMPUTE), default="auto")
    ap.add_argument("--alpha", type=float, default=1.0)
    ap.add_argument("--beta", type=float, default=0.0)
    ap.add_argument("--passes", type=int, default=1)
    ap.add_argument("--cache-target-mib", type=int, default=0, help="0: free memory at open")
    ap.add_argument("--chunk-mib", type=int, default=64)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--report", default=None, help="write the JSON report here")
    a = ap.parse_args()
    rep = run(a.m, a.n, a.k, int(a.op_a == "t"), int(a.op_b == "t"), a.dtype, a.c_dtype,
              a.compute, a.alpha, a.beta, a.passes, a.cache_target_mib << 20, a.chunk_mib << 20,
              a.device)
    if a.report:
        Path(a.report).write_text(json.dumps(rep, indent=1) + "\n")
    w = rep["workloads"][0]
    print(json.dumps({"status": rep["outcome"]["status"], "tiles": rep["plans"][0]["tile_count"],
                      "gemm_ms": rep["telemetry"]["gemm_timing"]["median_ms"],
                      "achieved_tflops": w["achieved_tflops"], "bytes_h2d": w["bytes_h2d"],
                      "all_results_match": rep["numerics"]["all_results_match"]}))
    raise SystemExit(rep["outcome"]["exit_code"])


if __name__ == "__main__":
    main()
