"""Times each call of a compat-table GEMM step (the bench's e2e step) separately.

    python -m xvram_b200.compat_phases --steps 83                   # strict FP32, C2
    python -m xvram_b200.compat_phases --steps 83 --budget-poll-ms 1000000000
    python -m xvram_b200.compat_phases --math 3                     # three-term TF32
    python -m xvram_b200.compat_phases --meminfo 2000               # cudaMemGetInfo latency

A step is memcpy H2D of A, B and C from pinned host memory, blas_sgemm, memcpy D2H of C,
through xvram_cuda_compat_get_api, with host wall-clock timing around every call.  It
prints one JSON line: the worst time of each call, the median step, the eight slowest
steps, and the runtime's deferred-GEMM and column-block counts.  `--budget-poll-ms`
overrides the session's budget poll interval (a huge value samples free memory once),
which separates budget-sampling stalls from the rest.  Set XVRAM_B200_SYNC_GEMM=1 in the
environment for the synchronous completion rule.  `--meminfo N` instead times N calls of
cudaMemGetInfo with the device idle and with GEMMs queued on another stream.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time


def meminfo_latency(calls: int) -> dict:
    import torch
    x = torch.randn(8192, 8192, device="cuda")
    side = torch.cuda.Stream()
    out = {}
    for label, busy in (("idle", False), ("busy", True)):
        lat = []
        for i in range(calls):
            if busy and i % 50 == 0:
                with torch.cuda.stream(side):
                    for _ in range(4):
                        x @ x
            t = time.perf_counter()
            torch.cuda.mem_get_info()
            lat.append(1e3 * (time.perf_counter() - t))
        torch.cuda.synchronize()
        lat.sort()
        out[label] = {"median_ms": lat[len(lat) // 2], "p99_ms": lat[int(0.99 * len(lat))],
                      "max_ms": lat[-1], "calls": calls}
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=6144)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--math", type=int, default=0, choices=[0, 2, 3],
                    help="blas_set_math_mode: 0 / 2 strict FP32, 3 three-term TF32")
    ap.add_argument("--budget-poll-ms", type=int, default=None)
    ap.add_argument("--meminfo", type=int, default=0,
                    help="time this many cudaMemGetInfo calls instead")
    a = ap.parse_args()

    if a.meminfo:
        print(json.dumps({"cudaMemGetInfo": meminfo_latency(a.meminfo)}))
        return

    import torch

    from xvram_b200 import compat as cp
    from xvram_b200 import device as xd

    m, n, k = a.m, a.n, a.k
    a_h = torch.empty((m, k), dtype=torch.float32).pin_memory()   # stored k x m (op T)
    b_h = torch.empty((n, k), dtype=torch.float32).pin_memory()   # stored k x n (op N)
    c_h = torch.empty((n, m), dtype=torch.float32).pin_memory()
    xd.fill_uniform(a_h, 10)
    xd.fill_uniform(b_h, 11)
    xd.fill_uniform(c_h, 12)
    c_out = torch.empty_like(c_h).pin_memory()

    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    if a.budget_poll_ms is not None:
        cfg.session.budget_poll_ms = a.budget_poll_ms
    api.check("initialize", api.initialize(cfg))
    h = api.blas_create()
    api.check("math", api.t.blas_set_math_mode(h, a.math))
    da, db, dc = api.malloc(a_h.nbytes), api.malloc(b_h.nbytes), api.malloc(c_h.nbytes)
    names = ("h2d_a", "h2d_b", "h2d_c", "sgemm", "d2h_c")
    calls = {key: [] for key in names}
    steps = []
    for i in range(a.warmup + a.steps):
        t = [time.perf_counter()]
        api.h2d(da, a_h.data_ptr(), a_h.nbytes)
        t.append(time.perf_counter())
        api.h2d(db, b_h.data_ptr(), b_h.nbytes)
        t.append(time.perf_counter())
        api.h2d(dc, c_h.data_ptr(), c_h.nbytes)
        t.append(time.perf_counter())
        api.check("sgemm", api.sgemm(h, 1, 0, m, n, k, 0.5, da, k, db, k, 1.5, dc, m))
        t.append(time.perf_counter())
        api.d2h(c_out.data_ptr(), dc, c_out.nbytes)
        t.append(time.perf_counter())
        if i >= a.warmup:
            for j, key in enumerate(names):
                calls[key].append(1e3 * (t[j + 1] - t[j]))
            steps.append(1e3 * (t[-1] - t[0]))
    info = cp.runtime_info()
    steps.sort()
    print(json.dumps({
        "m": m, "n": n, "k": k, "op": "TN", "math_mode": a.math, "steps": a.steps,
        "sync_gemm": os.environ.get("XVRAM_B200_SYNC_GEMM", "0") == "1",
        "budget_poll_ms": int(cfg.session.budget_poll_ms),
        "step_ms_median": statistics.median(steps),
        "slowest_steps_ms": [round(x, 2) for x in steps[-8:]],
        "call_ms_max": {key: round(max(v), 3) for key, v in calls.items()},
        "call_ms_median": {key: round(statistics.median(v), 3) for key, v in calls.items()},
        "gemm_deferred": int(info.gemm_deferred),
        "gemm_column_blocks": int(info.gemm_column_blocks)}))
    for d in (da, db, dc):
        api.free(d)
    api.blas_destroy(h)
    api.shutdown()


if __name__ == "__main__":
    main()
