#!/usr/bin/env python3
"""Benchmark of the out-of-core FP32 SGEMM path (one JSON line on rank 0).

Workload (the metric's single-GPU configuration): column-major
SGEMM M=8192 N=6144 K=4096, op(A)=T, op(B)=N, alpha=0.5, beta=1.5, A/B/C uniform[-1,1)
from seeds 10/11/12 (synthetic; no dataset).  N GPUs run one such problem each (weak
scaling: the C rows of the N-GPU job are split by rank, every rank owns an 8192-row
block and its A rows; B is shared: the kernel-only leg keeps a copy per GPU, the sharded
end-to-end leg reads 1/N of B per rank from the host and all-gathers it over NVLink).

  value   kernel-only TFLOP/s: the sm_100a SGEMM kernel on HBM-resident operands,
          K launches timed with CUDA events on the launching stream, max over ranks.
          The 416 MiB working set is larger than the 126 MB L2, so no flush is needed.
  e2e     the same metric through the reference-facing C ABI (xvram_cuda_compat_get_api):
          per step memcpy(H2D) of A, B, C from pinned host buffers, blas_sgemm, and
          memcpy(D2H) of C -- exactly what a reference caller does.
  roofline  achieved kernel TFLOP/s against the FP32 pipe peak measured in the same run:
          the higher of the scalar FFMA and packed FFMA2 probes (xvram_b200_ffma_probe,
          xvram_b200_ffma2_probe); `traffic` comes from the committed ncu
          summary profiles/sgemm_ffma_c2_traffic.json when present.
  host_link  pinned H2D/D2H GB/s measured here with every rank copying at once; the e2e
          roofline is max(FLOP / P_fp32, operand bytes / BW_host).
  cpu_baseline  the reference's CPU FP64 GEMM (reference_result, compiled from the
          reference sources into oracle/_ref) -- or the oracle port when that build is
          absent -- timed on a bounded sample on all host cores.

`--impl reference` times only that CPU implementation (the reference has no runnable
GPU path here: it needs CUDA 13, nvCOMP and cuBLAS 13 redistributables).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M, N, K = 8192, 6144, 4096
OP_A, OP_B = 1, 0
ALPHA, BETA = 0.5, 1.5
FLOP = 2.0 * M * N * K
WORKLOAD = "C2: column-major SGEMM M=8192 N=6144 K=4096 op(A)=T op(B)=N alpha=0.5 beta=1.5"
METRIC = "out-of-core SGEMM TFLOP/s + host-link GB/s vs roofline at 1/2/4/8 B200"


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# --------------------------------------------------------------------------- CPU legs
def cpu_reference_rate(threads: int, target_s: float):
    """Times the reference's own CPU FP64 GEMM (compat_bench reference_result, full k loop)
    on a bounded sample of C2's outputs; falls back to the oracle port over arrays."""
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle_lib import load_oracle, load_reference
    ref = load_reference()
    if ref is not None:
        def run(count, first=0):
            t0 = time.perf_counter()
            ref.xr_cpu_gemm_sample(M, N, K, first, count, ALPHA, BETA, 0, threads)
            return time.perf_counter() - t0
        kind = "reference"
        desc = "reference compat_bench reference_result (FP64, full K) over C2 outputs"
    else:
        import numpy as np
        orc = load_oracle()
        a = orc.uniform(K * M, 10)
        b = orc.uniform(K * N, 11)
        c = orc.uniform(M * N, 12)

        def run(count, first=0):
            idx = np.arange(first, first + count, dtype=np.int64) % (M * N)
            t0 = time.perf_counter()
            orc.gemm_sampled(OP_A, OP_B, K, ALPHA, a, K, b, K, BETA, c, M, idx % M, idx // M,
                             threads=threads)
            return time.perf_counter() - t0
        kind = "port"
        desc = "oracle FP64 port (xo_gemm_f64_sampled) over C2 outputs"
    run(4096)                       # thread start-up and first-touch out of the estimate
    probe = 1 << 19
    dt = max(run(probe), 1e-4)
    count = int(min(M * N, max(probe, probe * target_s / dt)))
    return kind, desc, run, count


def cpu_baseline_obj(threads: int, target_s: float = 40.0) -> dict:
    """The whole C2 output (50.3 M outputs, 412 GFLOP) when the host does it within
    `target_s` by a 512 Ki-output probe (about 11 s on 16 cores), else the largest sample
    that fits."""
    kind, desc, run, count = cpu_reference_rate(threads, target_s)
    dt = run(count)
    flop = 2.0 * K * count
    whole = "all" if count == M * N else f"a sample of {count}"
    return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
            "sample": f"{desc}: {whole} of {M * N} outputs ({flop / 1e9:.1f} GFLOP) in "
                      f"{dt:.1f} s"}


def run_reference_arm(args) -> None:
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    kind, desc, run, count = cpu_reference_rate(threads, target_s=2.0)
    for _ in range(args.warmup):
        run(count)
    times = [run(count) for _ in range(args.steps)]
    total = sum(times)
    value = 2.0 * K * count * args.steps / total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_outputs_per_step": count,
                   "note": "reference CPU FP64 GEMM on host cores (no GPU path builds here)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"{desc}: {count} outputs per step"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- clocks
INTERVAL_MS = 50


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs.

    The sampler is live and settled before the region starts: entering waits (up to 10 s)
    for nvidia-smi's second line (its start-up, which takes driver locks, is over by
    then), and leaving waits (up to 2 s) for one line after the region, so even a region
    shorter than the sampling interval is bracketed by samples.  `summary` uses the
    samples taken inside the region, or the two that bracket it when the region fell
    between samples.  Long workloads that map and unmap device memory throughout (the
    out-of-core and MLP runs) sample every 200 ms rather than every 50 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    def __init__(self, gpu_index: int, interval_ms: int = INTERVAL_MS):
        self.gpu = gpu_index
        self.interval_ms = interval_ms
        self.proc = None
        self.samples: list[tuple[float, str]] = []
        self.t_begin = self.t_end = 0.0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.monotonic() + 10.0
            while (len(self.samples) < 2 and time.monotonic() < deadline and
                   self.proc.poll() is None):
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.t_begin = time.monotonic()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), line.strip()))

    def __exit__(self, *exc):
        self.t_end = time.monotonic()
        if self.proc:
            deadline = self.t_end + 2.0
            while (time.monotonic() < deadline and self.proc.poll() is None and
                   not any(t >= self.t_end for t, _ in self.samples)):
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    @staticmethod
    def _parse(line: str):
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 9:
            return None
        try:
            sm, smax = float(parts[1]), float(parts[2])
        except ValueError:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        active = {n for n, v in zip(names, parts[5:9]) if v.lower().startswith("active")}
        return sm, smax, active

    def summary(self) -> dict:
        parsed = [(t, r) for t, r in ((t, self._parse(l)) for t, l in self.samples) if r]
        inside = [r for t, r in parsed if self.t_begin <= t <= self.t_end]
        how = "inside the timed region"
        if not inside:
            before = [r for t, r in parsed if t < self.t_begin][-1:]
            after = [r for t, r in parsed if t > self.t_end][:1]
            inside = before + after
            how = "bracketing the timed region (shorter than the sampling interval)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [r[0] for r in inside]
        smax = max(r[1] for r in inside)
        reasons = set().union(*(r[2] for r in inside))
        loaded = [x for x in sm if x > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "sampled": how,
                "region_ms": round(1e3 * (self.t_end - self.t_begin), 1),
                "interval_ms": self.interval_ms}


# ---------------------------------------------------------------- out-of-core workloads
def _rows_of(seed: int, n: int, first: int, count: int) -> "np.ndarray":
    """Rows [first, first + count) across all n columns of the n x n column-major matrix
    drawn from `seed` (element (i, k) is draw i + k n of the counter-based stream), as a
    (count, n) float64 array -- recomputed, not read back."""
    import numpy as np
    from xvram_b200 import device as xd
    out = np.empty((n, count), np.float32)
    for kk in range(n):
        xd.fill_uniform(out[kk], seed, first_index=first + kk * n, threads=1)
    return out.T.astype(np.float64)


def ooc_compat_leg(n: int, budget_gib: float, steps: int, peak_tflops: float, h2d_gbs: float,
                   d2h_gbs: float, device_ordinal: int = 0, tf32_steps: int = 0,
                   warmup: int = 0) -> dict:
    """One or more streamed GEMMs through the compat ABI with operands far above the device
    budget (BASELINE config 3's form: NT, alpha 1, beta 1, n^3, cache_target_bytes =
    budget): the operands are written through memcpy(H2D) into the adapter's host backing
    (256 MiB at a time, no full host copies), then each blas_sgemm call is timed on the host
    clock up to its completion (XVRAM_B200_SYNC_GEMM is not needed: a streamed GEMM
    completes before the call returns).  `warmup` untimed calls come first (the first call
    of a process also creates the frame pool; later calls remap its frames).  Parity: a 64 x 64 block of C is read back and checked
    against an FP64 recomputation of the same block from the seeded generators.
    With tf32_steps, that many more calls follow with the handle in math mode 3 (the
    three-term TF32 tensor-core path, FP32-accurate within the same tolerance), reported
    under "tf32x3" against max(TF32 work / the tensor peak, host bytes / the link)."""
    import numpy as np

    from xvram_b200 import compat as cp
    from xvram_b200 import device as xd

    seeds = (100, 101, 102)
    budget = int(budget_gib * (1 << 30))
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.cache_target_bytes = budget
    cfg.session.device_ordinal = device_ordinal
    api.check("initialize", api.initialize(cfg))
    stage = np.empty(64 << 20, np.float32)
    ptrs = []
    t_fill = time.perf_counter()
    for seed in seeds:
        d = api.malloc(n * n * 4)
        for off in range(0, n * n, stage.size):
            cnt = min(stage.size, n * n - off)
            xd.fill_uniform(stage[:cnt], seed, first_index=off)
            api.h2d(d + 4 * off, stage.ctypes.data, 4 * cnt)
        ptrs.append(d)
    t_fill = time.perf_counter() - t_fill
    del stage
    h = api.blas_create()
    flop = 2.0 * n ** 3
    for _ in range(warmup):
        api.check("sgemm", api.sgemm(h, 0, 1, n, n, n, 1.0, ptrs[0], n, ptrs[1], n, 1.0,
                                     ptrs[2], n))
        api.check("synchronize", api.t.synchronize())
    times, moved = [], []
    with ClockSampler(device_ordinal, 200) as clocks:
        for _ in range(max(steps, 1)):
            t0 = api.telemetry().runtime
            b0 = (t0.bytes_h2d, t0.bytes_d2h)
            start = time.perf_counter()
            api.check("sgemm", api.sgemm(h, 0, 1, n, n, n, 1.0, ptrs[0], n, ptrs[1], n, 1.0,
                                         ptrs[2], n))
            api.check("synchronize", api.t.synchronize())
            times.append(time.perf_counter() - start)
            t1 = api.telemetry().runtime
            moved.append((t1.bytes_h2d - b0[0], t1.bytes_d2h - b0[1]))
    strict_info = cp.runtime_info()
    tf32_times, tf32_moved = [], []
    if tf32_steps:
        api.check("math", api.t.blas_set_math_mode(h, 3))
        for _ in range(tf32_steps):
            t0 = api.telemetry().runtime
            b0 = (t0.bytes_h2d, t0.bytes_d2h)
            start = time.perf_counter()
            api.check("sgemm", api.sgemm(h, 0, 1, n, n, n, 1.0, ptrs[0], n, ptrs[1], n, 1.0,
                                         ptrs[2], n))
            api.check("synchronize", api.t.synchronize())
            tf32_times.append(time.perf_counter() - start)
            t1 = api.telemetry().runtime
            tf32_moved.append((t1.bytes_h2d - b0[0], t1.bytes_d2h - b0[1]))
        api.check("math", api.t.blas_set_math_mode(h, 0))
    tf32_info = cp.runtime_info()
    # parity on a 64 x 64 block (C = C0 + calls * A B^T in exact arithmetic)
    s, i0, j0 = 64, (n // 3) // 64 * 64, (2 * n // 3) // 64 * 64
    got = np.empty((s, s), np.float32)                       # [j, i]
    for jj in range(s):
        api.d2h(got[jj].ctypes.data, ptrs[2] + 4 * (i0 + (j0 + jj) * n), 4 * s)
    a_rows = _rows_of(seeds[0], n, i0, s)                    # A[i0.., :]
    b_rows = _rows_of(seeds[1], n, j0, s)                    # op(B)[:, j0..] = B[j0.., :]^T
    c0 = np.empty((s, s), np.float32)
    for jj in range(s):
        xd.fill_uniform(c0[jj], seeds[2], first_index=i0 + (j0 + jj) * n, threads=1)
    calls = warmup + len(times) + len(tf32_times)
    want = c0.astype(np.float64).T + calls * (a_rows @ b_rows.T)   # [i, j]
    err = float(np.max(np.abs(got.T.astype(np.float64) - want))) / (calls * n)
    tel = api.telemetry()
    info = strict_info
    for d in ptrs:
        api.free(d)
    api.blas_destroy(h)
    api.shutdown()
    sec = min(times)
    h2d_b, d2h_b = moved[times.index(sec)]
    alg_h2d = 3 * n * n * 4          # A + B + C_in, each once
    alg_d2h = n * n * 4              # C_out
    t_fp32 = flop / (peak_tflops * 1e12)
    t_roof = max(t_fp32, alg_h2d / (h2d_gbs * 1e9), alg_d2h / (d2h_gbs * 1e9))
    rt = tel.runtime
    out = {
        "workload": f"C3 form, out of core through the compat ABI: {n}^3 NT alpha 1 beta 1, "
                    f"{n * n * 4 >> 30} GiB per operand, device budget {budget_gib:g} GiB, 1 GPU",
        "value": flop / sec / 1e12, "unit": "TFLOP/s", "steps": len(times), "warmup": warmup,
        "ms_per_step": 1e3 * sec, "step_ms": [round(1e3 * t, 1) for t in times],
        "operand_bytes_over_budget": 3 * n * n * 4 / budget,
        "roofline": {"t_roof_ms": 1e3 * t_roof, "frac": t_roof / sec,
                     "bound": "fp32" if t_fp32 >= alg_h2d / (h2d_gbs * 1e9) else "host-link",
                     "p_fp32_tflops": peak_tflops, "h2d_gbs": h2d_gbs, "d2h_gbs": d2h_gbs},
        "host_link": {"h2d_bytes": h2d_b, "d2h_bytes": d2h_b, "algorithmic_h2d_bytes": alg_h2d,
                      "h2d_over_algorithmic": h2d_b / alg_h2d,
                      "achieved_h2d_gbs": h2d_b / sec / 1e9,
                      "achieved_d2h_gbs": d2h_b / sec / 1e9},
        "plan": {"block_m": int(info.last_block_m), "block_n": int(info.last_block_n),
                 "panel_k": int(info.last_panel_k), "steps": int(info.last_steps),
                 "panel_slots": int(info.last_panel_slots)},
        "residency": {"gemm_streamed": int(info.gemm_streamed),
                      "gemm_in_place": int(info.gemm_in_place),
                      "cache_target_bytes": int(rt.cache_target_bytes),
                      "resident_bytes_peak": int(rt.resident_bytes_peak),
                      "clean_evictions": int(rt.clean_evictions),
                      "dirty_evictions": int(rt.dirty_evictions),
                      "handle_reuses": int(rt.handle_reuses),
                      "mappings": int(rt.mappings), "unmaps": int(rt.unmaps),
                      "event_boundaries": int(rt.event_boundaries),
                      "maps_equal_unmaps": int(rt.mappings) == int(rt.unmaps),
                      "panel_slot_refills": int(info.panel_slot_refills),
                      "counters_note": "evictions and handle reuses count VMM unmaps and "
                                       "remaps, as the reference's do; a streamed GEMM "
                                       "refills the panel slots of its mapped frame arena "
                                       "in place (panel_slot_refills)",
                      "tiles_retired": int(tel.tiles_retired)},
        "check": {"block": [i0, j0, s], "max_abs_err_over_k_vs_fp64": err,
                  "within_1e-6": err <= 1e-6},
        "setup_s": {"fill_and_memcpy_h2d": round(t_fill, 1)},
        "clocks": clocks.summary(),
    }
    if tf32_times:
        tsec = min(tf32_times)
        th2d, td2h = tf32_moved[tf32_times.index(tsec)]
        p_tf32 = measured_tf32_peak()
        t_tensor = 3 * flop / (p_tf32 * 1e12)
        t_link = max(alg_h2d / (h2d_gbs * 1e9), alg_d2h / (d2h_gbs * 1e9))
        out["tf32x3"] = {
            "what": "the same call with blas_set_math_mode(3): three-term TF32 on "
                    "tcgen05/TMEM, within max|err|/(K max|a| max|b|) <= 1e-6 (the check "
                    "above covers both calls)",
            "value": flop / tsec / 1e12, "unit": "TFLOP/s", "ms_per_step": 1e3 * tsec,
            "roofline": {"t_roof_ms": 1e3 * max(t_tensor, t_link),
                         "frac": max(t_tensor, t_link) / tsec,
                         "bound": "tensor" if t_tensor >= t_link else "host-link",
                         "p_tf32_tflops": p_tf32, "tf32_flop": 3 * flop},
            "host_link": {"h2d_bytes": th2d, "d2h_bytes": td2h,
                          "h2d_over_algorithmic": th2d / alg_h2d,
                          "achieved_h2d_gbs": th2d / tsec / 1e9},
            "plan": {"block_m": int(tf32_info.last_block_m),
                     "block_n": int(tf32_info.last_block_n),
                     "panel_k": int(tf32_info.last_panel_k),
                     "steps": int(tf32_info.last_steps)},
        }
    return out


def ooc_sharded_leg(Mt: int, Nt: int, Kt: int, steps: int, warmup: int, world: int, rank: int,
                    local: int, dev, barrier, max_over_ranks, peak: float, h2d: float,
                    d2h: float) -> dict:
    """BASELINE config 4's form (NN, beta 0, C rows sharded over the GPUs, B read from the
    host once per node and all-gathered over NVLink) as one fixed total problem split over
    however many ranks run it (strong scaling).  Each step is one xvram_b200_sgemm_sharded
    call from pinned host memory to pinned host memory, timed between barriers, max over
    ranks; rows per rank from xvram_b200_shard_rows.  Every rank returns the same dict."""
    import numpy as np
    import torch

    from xvram_b200 import device as xd
    from xvram_b200 import shard

    r0, mr = shard.rows(Mt, world, rank)
    m_max = max(shard.rows(Mt, world, q)[1] for q in range(world))
    # op N operands: A_local is mr x K (rows r0.. of the seeded M x K matrix), B is K x N.
    # Allocated page-locked directly (no pageable copy first: full C4's C is 256 GiB).
    a_h = torch.empty((Kt, max(mr, 1)), dtype=torch.float32, pin_memory=True)  # mr x K, col-major
    b_h = torch.empty((Nt, Kt), dtype=torch.float32, pin_memory=True)          # K x N, col-major
    c_h = torch.empty((Nt, max(mr, 1)), dtype=torch.float32, pin_memory=True)  # mr x N, col-major
    if mr:
        threads = 0 if mr >= (1 << 17) else 1   # all host threads only for long columns
        for kk in range(Kt):  # A_local column k holds rows r0..r0+mr of column k
            xd.fill_uniform(a_h[kk, :mr], 40, first_index=kk * Mt + r0, threads=threads)
    # B: every rank holds the whole K x N matrix but copies only its 1/P column slice of
    # each C block to the GPU (the others arrive over NVLink).  With several ranks the rank
    # fills just those columns, plus the columns of its sampled checks (the generator is
    # counter-based, so every rank writes the same values into a column it fills).
    rng = np.random.default_rng(rank)
    samples = list(zip(rng.integers(0, max(mr, 1), 16), rng.integers(0, Nt, 16)))
    if world == 1:
        xd.fill_uniform(b_h, 41)
    else:
        # the library's block width (xvram_b200_sgemm_sharded's default is 576 columns;
        # checked against the call's plan after the first step)
        nb = min(Nt, -(-env_int("XVRAM_B200_SHARD_BLOCK_N", 576) // 32) * 32)
        wc = -(-nb // world)
        cols = {int(c) for _, c in samples}
        for n0 in range(0, Nt, nb):
            cols.update(range(n0 + rank * wc, min(n0 + (rank + 1) * wc, n0 + nb, Nt)))
        for j in sorted(cols):
            xd.fill_uniform(b_h[j], 41, first_index=j * Kt, threads=1)
    uid = shard.exchange_unique_id(rank) if world > 1 else shard.unique_id()
    group = shard.ShardGroup(uid, rank, world)

    def step():
        st = group.sgemm(0, 0, mr, Nt, Kt, 1.0, a_h, max(mr, 1), b_h, Kt, 0.0, c_h,
                         max(mr, 1), panel_k=2048)
        assert st == 0, st

    for _ in range(warmup):
        step()
    if world > 1 and warmup:
        assert group.last_plan()["block_n"] == nb, (group.last_plan()["block_n"], nb)
    times = []
    with ClockSampler(local, 200) as clocks:
        for _ in range(steps):
            barrier()
            t0 = time.perf_counter()
            step()
            barrier()
            times.append(max_over_ranks(time.perf_counter() - t0))
    plan = group.last_plan()
    group.close()
    # sampled check: 16 outputs of this rank against FP64 (the operands' generator is
    # counter-based, so any element can be recomputed)
    worst = 0.0
    if mr > 0:
        for r, c in samples:
            ref = float(a_h[:, int(r)].double().numpy() @ b_h[int(c)].double().numpy())
            worst = max(worst, abs(float(c_h[int(c), int(r)]) - ref) / Kt)
    worst = max_over_ranks(worst)
    h2d_moved = max_over_ranks(float(plan["h2d_bytes"]))
    sec = statistics.median(times)
    flop = 2.0 * Mt * Nt * Kt
    t_compute = flop / world / (peak * 1e12)
    h2d_rank = 4.0 * (m_max * Kt + Kt * Nt / world)   # A rows + a 1/P share of B, once
    d2h_rank = 4.0 * m_max * Nt
    t_roof = max(t_compute, h2d_rank / (h2d * 1e9), d2h_rank / (d2h * 1e9))
    del a_h, b_h, c_h
    return {
        "workload": f"C4 form, strong-scaled: {Mt} x {Nt} x {Kt} NN beta 0, C rows over "
                    f"{world} GPU(s), B from host once per node + NCCL all-gather",
        "value": flop / sec / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": 1e3 * sec, "scaling": "strong",
        "step_ms": [round(1e3 * t, 2) for t in times],
        "roofline": {"t_roof_ms": 1e3 * t_roof, "frac": t_roof / sec, "per": "rank",
                     "p_fp32_tflops_per_gpu": peak, "h2d_gbs_concurrent": h2d,
                     "d2h_gbs_concurrent": d2h,
                     "bound": "fp32" if t_compute >= max(h2d_rank / (h2d * 1e9),
                                                         d2h_rank / (d2h * 1e9)) else "host-link"},
        "host_link": {"h2d_bytes_per_rank_max": h2d_moved,
                      "h2d_over_algorithmic": h2d_moved / h2d_rank,
                      "d2h_bytes_per_rank": d2h_rank},
        "plan": {key: plan[key] for key in ("row_groups", "group_rows", "block_n", "panel_k",
                                            "gathers", "device_bytes")},
        "check": {"sampled_outputs_per_rank": 16, "max_abs_err_over_k_vs_fp64": worst,
                  "within_1e-6": worst <= 1e-6},
        "clocks": clocks.summary(),
    }


def child_c3s(args, local: int) -> dict:
    """`bench.py --workload c3s --steps 1` in a child process; its JSON line as a dict."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--workload", "c3s", "--steps", "1",
           "--warmup", "1", "--ooc-n", str(args.ooc_n), "--ooc-budget-gib",
           str(args.ooc_budget_gib), "--ooc-tf32-steps", "1"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", str(local)))
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(key, None)
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=1200)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"error": f"rc {r.returncode}: {(r.stderr or r.stdout)[-400:]}"}
    out = json.loads(lines[-1])
    for key in ("metric", "n_gpus", "dtype", "data"):
        out.pop(key, None)
    return out


def run_out_of_core(args) -> None:
    """--workload c3s: the compat out-of-core leg alone (n = --ooc-n, budget
    --ooc-budget-gib), printed as one JSON line."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(device=dev)
    peak_tflops, probes = measure_fp32_peak(dev, stream)
    h2d_gbs, d2h_gbs = measure_link(dev, stream, lambda: None)
    leg = ooc_compat_leg(args.ooc_n, args.ooc_budget_gib, args.steps, peak_tflops, h2d_gbs,
                         d2h_gbs, tf32_steps=args.ooc_tf32_steps, warmup=args.warmup)
    leg["roofline"]["fp32_probes"] = probes
    print(json.dumps({"metric": METRIC, "n_gpus": 1, "dtype": "f32", "data": "synthetic",
                      **leg}), flush=True)


def run_sharded_c4(args) -> None:
    """--workload c4s: the strong-scaled C4-form leg alone (--c4-m x --c4-n x --c4-k)."""
    import datetime

    import torch
    import torch.distributed as dist

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://",
                                timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.Stream(device=dev)
    peak, probes = measure_fp32_peak(dev, stream)
    h2d, d2h = measure_link(dev, stream, barrier)
    h2d, d2h = -max_over_ranks(-h2d), -max_over_ranks(-d2h)
    leg = ooc_sharded_leg(args.c4_m, args.c4_n, args.c4_k, args.steps, args.warmup, world, rank,
                          local, dev, barrier, max_over_ranks, peak, h2d, d2h)
    leg["roofline"]["fp32_probes"] = probes
    if rank == 0:
        print(json.dumps({"metric": METRIC, **leg}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------- MLP workload (C5)
def run_mlp(args) -> None:
    """BASELINE config 5 through the SDK (include/xvram.h): 24 x Linear(16384 -> 16384,
    bias) + ReLU, batch 512, weights N(0, 1/16384), input uniform[-1,1], device budget
    8 GiB per GPU.  The weights live in the session's pinned host backing; every forward
    streams each layer's weight through the frame cache.  Per layer the host submits, in
    order: prefetch of the next layer's weight, the GEMM (strict FP32), and a transaction
    whose callback runs bias + ReLU on the resident output, then waits only at the end.
    Activations are column-major features x batch (= row-major batch x features); weights
    are stored column-major out x in, so op(A) = N.  A step is one forward pass including
    the input upload and the output download.

    Under torchrun (N > 1) each layer is split by output features (xvram_b200.mlp.
    ShardedMLP): rank r streams rows [r F/N, (r + 1) F/N) of every weight from its host
    memory, and the activation row blocks are all-gathered over NVLink between layers;
    strong scaling (the same 24-layer forward on N GPUs), time = max over ranks."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from xvram_b200 import sdk
    from xvram_b200 import shard
    from xvram_b200.mlp import ShardedMLP, StreamedMLP

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://",
                                timeout=datetime.timedelta(seconds=300))
    F, BATCH, LAYERS = args.mlp_features, args.mlp_batch, args.mlp_layers
    if F % world:
        raise SystemExit("features must divide evenly over the GPUs")
    Fr = F // world
    rows = slice(rank * Fr, (rank + 1) * Fr)
    budget = int(args.mlp_budget_gib * (1 << 30))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.Stream(device=dev)
    peak_tflops, probes = measure_fp32_peak(dev, stream)
    h2d_gbs, d2h_gbs = measure_link(dev, stream, barrier)
    h2d_gbs, d2h_gbs = -max_over_ranks(-h2d_gbs), -max_over_ranks(-d2h_gbs)
    wbytes = Fr * F * 4
    abytes = F * BATCH * 4

    def weight(i):  # column-major out x in, N(0, 1/F), regenerated on demand for the check
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + i)
        return torch.randn((F, F), generator=g, device=dev) / np.sqrt(F)  # [in][out] = col-major

    g = torch.Generator(device=dev)
    g.manual_seed(999)
    bias_all = ((torch.rand((LAYERS, F), generator=g, device=dev) * 2 - 1) / np.sqrt(F))
    x = (torch.rand((BATCH, F), generator=g, device=dev) * 2 - 1)

    # the sharded layers' exchange uses an F x B staging workspace in each transaction.
    # LRU: while layer i computes, the prefetch of layer i+1's weight takes the frames of
    # layer i-1 (least recently used), never those of the weight still in use.
    s = sdk.Sdk(sdk.session_config(device_ordinal=local, cache_target_bytes=budget,
                                   workspace_cap_bytes=max(4 << 20, abytes),
                                   cache_policy=sdk.CACHE_POLICY_LRU))
    group = None
    if world > 1:
        group = shard.ShardGroup(shard.exchange_unique_id(rank), rank, world)
        net = ShardedMLP(s, group, F, BATCH, LAYERS)
    else:
        net = StreamedMLP(s, F, BATCH, LAYERS)
    stage = torch.empty(Fr * F, dtype=torch.float32).pin_memory()
    for i in range(LAYERS):
        # weight(i) is [in][out]: this rank's out-rows are its columns -> [in][Fr] block
        stage.copy_(weight(i)[:, rows].contiguous().reshape(-1))
        net.load_weight(i, stage)
    del stage
    net.load_biases(bias_all[:, rows].cpu().contiguous().pin_memory())
    x_h = x.cpu().contiguous().pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()

    def forward():
        net.forward(x_h, out_h)

    for _ in range(args.warmup):
        forward()
    barrier()
    times = []
    t0 = s.telemetry()
    with ClockSampler(local, 200) as clocks:
        for _ in range(args.steps):
            barrier()
            start = time.perf_counter()
            forward()
            times.append(max_over_ranks(time.perf_counter() - start))
    t1 = s.telemetry()
    assert net.statuses and all(st == 0 for st in net.statuses)

    # FP64 check of sampled batch rows against the same weights (regenerated on the GPU)
    cols = [0, 1, BATCH // 2, BATCH - 1]
    ref = x[cols].double()
    for i in range(LAYERS):
        ref = torch.relu(ref @ weight(i).double() + bias_all[i].double())
    got = out_h[cols].to(dev).double()
    err = max_over_ranks(float((got - ref).abs().max()))
    scale = float(ref.abs().max())

    sec = statistics.median(times)
    flop = LAYERS * 2.0 * F * F * BATCH
    h2d_moved = (t1.bytes_h2d - t0.bytes_h2d) / args.steps
    # per rank: its weight rows, input, bias slices, once each
    alg_h2d = LAYERS * wbytes + abytes + LAYERS * Fr * 4
    alg_d2h = abytes
    t_roof = max(flop / world / (peak_tflops * 1e12), alg_h2d / (h2d_gbs * 1e9),
                 alg_d2h / (d2h_gbs * 1e9))
    net.close()
    tel = s.telemetry()
    s.close()
    if group is not None:
        group.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "workload": f"C5: {LAYERS} x Linear({F}->{F}, bias) + ReLU, batch {BATCH}, "
                    f"device budget {args.mlp_budget_gib} GiB per GPU, through the SDK "
                    f"(xvram_get_api)" + (f"; layers split by output features over {world} "
                                          "GPUs, activations all-gathered over NVLink"
                                          if world > 1 else ""),
        "value": flop / sec / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * sec, "higher_is_better": True,
        "scaling": "strong", "dtype": "f32",
        "data": "synthetic (seeded torch generators on the GPU)",
        "roofline": {"t_roof_ms": 1e3 * t_roof, "frac": t_roof / sec,
                     "bound": "host-link" if alg_h2d / (h2d_gbs * 1e9) >
                     flop / world / (peak_tflops * 1e12) else "fp32",
                     "p_fp32_tflops": peak_tflops, "fp32_probes": probes, "h2d_gbs": h2d_gbs,
                     "d2h_gbs": d2h_gbs, "per": "rank"},
        "host_link": {"h2d_bytes_per_step_rank0": h2d_moved,
                      "algorithmic_h2d_bytes_per_rank": alg_h2d,
                      "achieved_h2d_gbs_rank0": h2d_moved / sec / 1e9,
                      "concurrent_ranks": world},
        "check": {"sampled_batch_rows": cols, "max_abs_err_vs_fp64": err,
                  "max_abs_ref": scale},
        "residency": {"cache_target_bytes": int(tel.cache_target_bytes),
                      "resident_bytes_peak": int(tel.resident_bytes_peak),
                      "clean_evictions": int(tel.clean_evictions),
                      "dirty_evictions": int(tel.dirty_evictions),
                      "handle_reuses": int(tel.handle_reuses), "mappings": int(tel.mappings),
                      "transactions_completed": int(tel.transactions_completed)},
        "step_ms": [1e3 * t for t in times],
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def measure_ffma_peak(dev, stream, iters: int = 8000, packed: bool = False) -> float:
    """FP32 pipe peak (TFLOP/s) from the FFMA probe (scalar FFMA, or packed FFMA2 with
    `packed`): ~15 ms launches, best of 7."""
    import torch
    from xvram_b200 import device as xd
    sink = torch.zeros(1, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 4
    best = 0.0
    with torch.cuda.stream(stream):
        for i in range(8):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            assert xd.ffma_probe(blocks, iters, sink, stream, packed=packed) == 0
            e1.record(stream)
            e1.synchronize()
            if i:
                best = max(best, 2.0 * blocks * 256 * iters * 512 / (e0.elapsed_time(e1) * 1e-3))
    return best / 1e12


def measure_fp32_peak(dev, stream) -> tuple[float, dict]:
    """The FP32 pipe peak as the higher of the scalar and packed probes (the SGEMM main
    loop issues packed FMAs), with both figures for the record."""
    scalar = measure_ffma_peak(dev, stream)
    packed = measure_ffma_peak(dev, stream, packed=True)
    return max(scalar, packed), {"ffma_probe": scalar, "ffma2_probe": packed}


def cublas_tf32_tflops(dev) -> float:
    """cuBLAS TF32 GEMM throughput measured here (8192^3, best of 5, CUDA events): the
    library ceiling for the tensor-core path, beside the BF16 / 2 figure below."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        for _ in range(2):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            e1.synchronize()
            best = max(best, 2.0 * n ** 3 / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        del a, b
        return best
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def library_sgemm_leg(dev, stream, A, B, c_h, steps: int, warmup: int, ours_ms: float) -> dict:
    """The reference's own contraction call on this GPU: cublasGemmEx with
    CUBLAS_COMPUTE_32F_PEDANTIC in pedantic math mode (xvram_b200.native_baseline), on the
    same resident operands and op pair as the headline step, timed the same way (warm-up,
    then `steps` calls between CUDA events on the same stream).  Also how far its C lies
    from this library's on the same inputs, as max|C_lib - C_ours| / (K max|a| max|b|):
    both are strict FP32 with different summation orders."""
    import torch
    from xvram_b200 import device as xd
    from xvram_b200.native_baseline import PedanticSgemm
    try:
        gemm = PedanticSgemm(stream.cuda_stream)
    except (RuntimeError, OSError, AttributeError) as e:
        return {"unavailable": str(e)}
    with gemm, torch.cuda.stream(stream):
        c0 = c_h.to(dev, non_blocking=False)
        c_lib = c0.clone()

        def call(c):
            gemm(OP_A, OP_B, M, N, K, ALPHA, A.data_ptr(), K, B.data_ptr(), K, BETA,
                 c.data_ptr(), M)

        for _ in range(max(3, warmup)):
            call(c_lib)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            call(c_lib)
        e1.record(stream)
        e1.synchronize()
        lib_ms = e0.elapsed_time(e1) / steps
        version = gemm.version()
        c_lib.copy_(c0)
        c_ours = c0.clone()
        call(c_lib)
        assert xd.sgemm(OP_A, OP_B, M, N, K, ALPHA, A, K, B, K, BETA, c_ours, M,
                        stream=stream) == 0
        scale = K * float(A.abs().max()) * float(B.abs().max())
        diff = float((c_lib - c_ours).abs().max()) / scale
        stream.synchronize()
        assert xd.kernel_status(stream) == 0
        del c0, c_lib, c_ours
    return {"what": "cublasGemmEx, CUBLAS_COMPUTE_32F_PEDANTIC, CUBLAS_PEDANTIC_MATH: the "
                    "reference's strict-FP32 contraction (src/gemm/executor.cpp:211-218, "
                    "src/platform/cublas/cublas_api.cpp:634-686) on the headline operands",
            "cublas_version": version,
            "value": FLOP / (lib_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": lib_ms,
            "ours_ms_per_step": ours_ms, "speedup_ours_over_library": lib_ms / ours_ms,
            "max_normalized_diff_vs_ours": diff}


def measured_tf32_peak():
    """Dense TF32 tensor peak implied by the driver-measured BF16 GEMM burst figure."""
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return peaks["bf16_tflops"] / 2.0
    except (OSError, ValueError, KeyError):
        return 1590.0 / 2.0  # fallback figure of the profiling recipe (bf16 1.59 PFLOP/s)


def measure_link(dev, stream, barrier) -> tuple[float, float]:
    """Pinned H2D and D2H GB/s per GPU (256 MiB copies, best of 4), every rank copying at
    the same time (a barrier before each copy), so shared root complexes show."""
    import torch
    probe_h = torch.empty(64 << 20, dtype=torch.float32).pin_memory()
    probe_d = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    h2d = d2h = 0.0
    with torch.cuda.stream(stream):
        for _ in range(4):
            e0, e1, e2, e3 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
            barrier()
            e0.record(stream)
            probe_d.copy_(probe_h, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            barrier()
            e2.record(stream)
            probe_h.copy_(probe_d, non_blocking=True)
            e3.record(stream)
            e3.synchronize()
            h2d = max(h2d, probe_h.nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
            d2h = max(d2h, probe_h.nbytes / (e2.elapsed_time(e3) * 1e-3) / 1e9)
    return h2d, d2h


# ------------------------------------------------------------------------------ GPU arm
def pipelined_steps(n, stream, side, bufs, gathered, consumed, gather, kernel) -> None:
    """n steps of (gather B into a buffer, kernel on it) with two B buffers: step i+1's
    gather runs on `side` while step i's kernel runs on `stream`.  The side stream waits
    for everything already on `stream` first (so a start event recorded there covers the
    first gather), and a buffer is refilled only after the kernel that read it.  The
    last kernel is the last work on `stream`."""
    import torch
    side.wait_stream(stream)

    def issue(i):
        buf = i % 2
        side.wait_event(consumed[buf])
        with torch.cuda.stream(side):
            gather(bufs[buf])
            gathered[buf].record(side)

    issue(0)
    for i in range(n):
        if i + 1 < n:
            issue(i + 1)
        stream.wait_event(gathered[i % 2])
        with torch.cuda.stream(stream):
            assert kernel(bufs[i % 2]) == 0
        consumed[i % 2].record(stream)


def main_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://",
                                timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    from xvram_b200 import compat as cp
    from xvram_b200 import device as xd
    from xvram_b200._native import lib

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Inputs: rank r owns C rows [8192 r, 8192 (r+1)) of the weak-scaled job; its A rows
    # and the B panel are generated from the same seeded streams (offset by rank).
    a_h = torch.empty((M, K), dtype=torch.float32).pin_memory()    # stored K x M (op T)
    b_h = torch.empty((N, K), dtype=torch.float32).pin_memory()    # stored K x N (op N)
    c_h = torch.empty((N, M), dtype=torch.float32).pin_memory()    # M x N
    xd.fill_uniform(a_h, 10, first_index=rank * M * K)
    xd.fill_uniform(b_h, 11)
    xd.fill_uniform(c_h, 12, first_index=rank * M * N)
    c_out = torch.empty_like(c_h).pin_memory()

    stream = torch.cuda.Stream(device=dev)
    A = a_h.to(dev)
    B = b_h.to(dev)
    Cd = c_h.to(dev)
    torch.cuda.synchronize()

    # FP32 pipe peak on this device, this run (FFMA probe), repeated after the kernel's
    # timed region so both see a warm clock; pinned host-link bandwidth.
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak_tflops, probes = measure_fp32_peak(dev, stream)
    h2d, d2h = measure_link(dev, stream, barrier)
    # the job's host link is as slow as its slowest GPU's
    h2d, d2h = -max_over_ranks(-h2d), -max_over_ranks(-d2h)

    # ---------------- kernel-only: inputs resident in HBM.  At N > 1 the job is one
    # problem split by C rows: each rank holds its A rows, its C rows and a 1/N column
    # slice of the shared B.  Every step all-gathers B over NVLink (NCCL) and runs the
    # kernel on the gathered B; B is double-buffered, so step i+1's gather (on a side
    # stream) overlaps step i's kernel, as a pipeline of successive GEMMs would run.
    B_slice = B[rank * (N // world):(rank + 1) * (N // world)].clone() if world > 1 else None
    B_run = torch.empty_like(B) if world > 1 else B
    if world > 1:
        assert N % world == 0

    def gather_b(dst):
        dist.all_gather_into_tensor(dst, B_slice)

    def launch_steps(n: int) -> None:
        """n steps on `stream` (and, at N > 1, its side stream); enqueue only."""
        if world == 1:
            with torch.cuda.stream(stream):
                for _ in range(n):
                    assert xd.sgemm(OP_A, OP_B, M, N, K, ALPHA, A, K, B, K, BETA, Cd, M,
                                    stream=stream) == 0
            return
        pipelined_steps(n, stream, side, B_bufs, gathered, consumed, gather_b,
                        lambda bb: xd.sgemm(OP_A, OP_B, M, N, K, ALPHA, A, K, bb, K, BETA, Cd,
                                            M, stream=stream))

    # high priority, so the gather's few CTAs are scheduled as soon as kernel CTAs retire
    side = torch.cuda.Stream(device=dev, priority=-1) if world > 1 else None
    B_bufs = [B_run, torch.empty_like(B)] if world > 1 else None
    gathered = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]

    launch_steps(args.warmup)
    torch.cuda.synchronize()
    assert xd.kernel_status(stream) == 0
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        launch_steps(args.steps)   # at N > 1 the first gather waits for `start` (below)
        stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    barrier()
    assert xd.kernel_status(stream) == 0
    peak_again, probes_again = measure_fp32_peak(dev, stream)
    peak_tflops = max(peak_tflops, peak_again)
    probes = {key: max(probes[key], probes_again[key]) for key in probes}
    step_ms = start.elapsed_time(stop) / args.steps
    step_ms_max = max_over_ranks(step_ms)
    value = world * FLOP / (step_ms_max * 1e-3) / 1e12
    # The dominant kernel alone (its launches timed on the same stream, no gather), for
    # the roofline: at N = 1 this is the step itself.
    if world > 1:
        k0e, k1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            k0e.record(stream)
            for _ in range(args.steps):
                assert xd.sgemm(OP_A, OP_B, M, N, K, ALPHA, A, K, B_run, K, BETA, Cd, M,
                                stream=stream) == 0
            k1e.record(stream)
        k1e.synchronize()
        kernel_ms = k0e.elapsed_time(k1e) / args.steps
    else:
        kernel_ms = step_ms
    achieved = FLOP / (kernel_ms * 1e-3) / 1e12
    del B_slice, B_bufs
    library = library_sgemm_leg(dev, stream, A, B, c_h, args.steps, args.warmup, kernel_ms)

    # ---------------- kernel-only, tensor-core path (three-term TF32 on tcgen05/TMEM)
    tc_need = lib.xvram_b200_sgemm_workspace_bytes(OP_A | 0x100, OP_B, M, N, K)
    tc_ws = torch.empty(tc_need // 4 + 64, dtype=torch.float32, device=dev)
    C_tc = Cd.clone()

    def launch_tc():
        st = xd.sgemm_ws(OP_A, OP_B, M, N, K, ALPHA, A, K, B, K, BETA, C_tc, M, tc_ws, tc_need,
                         stream=stream, path=3)
        assert st == 0, st

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            launch_tc()
    stream.synchronize()
    barrier()
    with ClockSampler(local) as tc_clocks:
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            t0e.record(stream)
            for _ in range(args.steps):
                launch_tc()
            t1e.record(stream)
        t1e.synchronize()
    assert xd.kernel_status(stream) == 0
    tc_ms = max_over_ranks(t0e.elapsed_time(t1e) / args.steps)
    del tc_ws, C_tc
    tf32_cublas = cublas_tf32_tflops(dev)

    # ---------------- end to end, sharded path: C rows per rank, B panels read 1/N per rank
    # from host memory and all-gathered over NVLink (xvram_b200_sgemm_sharded)
    from xvram_b200 import shard
    uid = shard.exchange_unique_id(rank) if world > 1 else shard.unique_id()
    group = shard.ShardGroup(uid, rank, world)
    c_sh = torch.empty_like(c_h).pin_memory()

    def sharded_step():
        c_sh.copy_(c_h)  # host-side reset of C (outside the device work, same every step)
        st = group.sgemm(OP_A, OP_B, M, N, K, ALPHA, a_h, K, b_h, K, BETA, c_sh, M, panel_k=1024)
        assert st == 0, st

    for _ in range(args.warmup):
        sharded_step()
    barrier()
    sh_times = []
    for _ in range(args.steps):
        c_sh.copy_(c_h)
        barrier()
        t0 = time.perf_counter()
        st = group.sgemm(OP_A, OP_B, M, N, K, ALPHA, a_h, K, b_h, K, BETA, c_sh, M, panel_k=1024)
        sh_times.append(time.perf_counter() - t0)
        assert st == 0, st
    sharded_s = max_over_ranks(sum(sh_times) / len(sh_times))
    group.close()
    sh_h2d = a_h.nbytes + b_h.nbytes // world + c_h.nbytes
    sh_d2h = c_h.nbytes

    # ---------------- end to end through the compat C ABI
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.device_ordinal = local
    api.check("initialize", api.initialize(cfg))
    h = api.blas_create()
    da, db, dc = api.malloc(a_h.nbytes), api.malloc(b_h.nbytes), api.malloc(c_h.nbytes)

    call_ms = {key: [] for key in ("h2d_a", "h2d_b", "h2d_c", "sgemm", "d2h_c")}

    def e2e_step():
        t = [time.perf_counter()]
        api.h2d(da, a_h.data_ptr(), a_h.nbytes)
        t.append(time.perf_counter())
        api.h2d(db, b_h.data_ptr(), b_h.nbytes)
        t.append(time.perf_counter())
        api.h2d(dc, c_h.data_ptr(), c_h.nbytes)
        t.append(time.perf_counter())
        api.check("sgemm", api.sgemm(h, OP_A, OP_B, M, N, K, ALPHA, da, K, db, K, BETA, dc, M))
        t.append(time.perf_counter())
        api.d2h(c_out.data_ptr(), dc, c_out.nbytes)
        t.append(time.perf_counter())
        for i, key in enumerate(call_ms):
            call_ms[key].append(1e3 * (t[i + 1] - t[i]))

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_marks = [t0]
    for _ in range(args.steps):
        e2e_step()
        e2e_marks.append(time.perf_counter())
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / args.steps
    barrier()
    e2e_s_max = max_over_ranks(e2e_s)
    e2e_step_ms = sorted(1e3 * (b - a) for a, b in zip(e2e_marks[:-1], e2e_marks[1:]))
    # per-call medians over the timed steps (the warm-up steps come first in each list)
    e2e_call_ms = {key: statistics.median(v[-args.steps:]) for key, v in call_ms.items()}
    trace_records = None
    if args.trace and rank == 0:
        # one more step, outside the timed region, in the reference's trace format
        from xvram_b200.report import TracedCompat
        with open(args.trace, "w") as sink:
            tr = TracedCompat(api, sink)
            tr.h2d(da, a_h.data_ptr(), a_h.nbytes)
            tr.h2d(db, b_h.data_ptr(), b_h.nbytes)
            tr.h2d(dc, c_h.data_ptr(), c_h.nbytes)
            api.check("sgemm", tr.sgemm(h, OP_A, OP_B, M, N, K, ALPHA, da, K, db, K, BETA, dc, M))
            tr.d2h(c_out.data_ptr(), dc, c_out.nbytes)
            tr.close()
            trace_records = tr.records
    tel = api.telemetry()
    info = cp.runtime_info()
    # the same steps with the handle in TF32 tensor-op math mode (three-term TF32 kernel)
    api.check("math", api.t.blas_set_math_mode(h, 3))
    for _ in range(args.warmup):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_tc_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    api.check("math", api.t.blas_set_math_mode(h, 0))
    tc_call_ms = {key: statistics.median(v[-args.steps:]) for key, v in call_ms.items()}
    tc_step_ms = sorted(sum(v[-args.steps:][i] for v in call_ms.values())
                        for i in range(args.steps))
    # the canonicalising transposes per in-place GEMM, plus its kernel, or one kernel per C
    # column block when the call returned before its kernels finished (the default)
    launches_e2e = (int(info.gemm_in_place) * (int(OP_A == 1) + int(OP_B == 0)) +
                    (int(info.gemm_column_blocks) or int(info.gemm_in_place)))
    for d in (da, db, dc):
        api.free(d)
    api.blas_destroy(h)
    api.shutdown()

    h2d_bytes = a_h.nbytes + b_h.nbytes + c_h.nbytes
    d2h_bytes = c_out.nbytes
    # e2e roofline per GPU: max(FP32 compute at the measured peak, operand bytes over the
    # measured pinned H2D bandwidth with every rank copying at once).  Operand bytes are
    # A + B + C_in + C_out once each; with B shared over NVLink a rank moves 1/N of B.
    t_compute = FLOP / (peak_tflops * 1e12)
    t_roof = max(t_compute, h2d_bytes / (h2d * 1e9) + d2h_bytes / (d2h * 1e9))
    t_roof_overlap = max(t_compute, (h2d_bytes + d2h_bytes) / (h2d * 1e9))
    t_roof_sharded = max(t_compute, (sh_h2d + sh_d2h) / (h2d * 1e9))
    # The floor the call sequence allows: cudaMemcpy returns only once its copy is done, so
    # the three H2D copies precede the GEMM in series; C's D2H can overlap the kernel.
    t_floor_api = h2d_bytes / (h2d * 1e9) + max(kernel_ms * 1e-3, d2h_bytes / (d2h * 1e9))

    # DRAM bytes per launch of the dominant kernel on this workload, from the committed ncu
    # capture of this bench's own TN launch (profiles/sgemm_ffma_c2_tn_traffic.json).
    traffic, traffic_source = None, None
    tfile = ROOT / "profiles" / "sgemm_ffma_c2_tn_traffic.json"
    if tfile.exists():
        try:
            tj = json.loads(tfile.read_text())
            traffic = tj.get("dram_bytes_per_launch")
            traffic_source = f"{tfile.relative_to(ROOT)}: {tj.get('kernel')} ({tj.get('command')})"
        except (ValueError, OSError):
            traffic = None

    # ---------------- out of core: the metric's own configurations, after the C2 legs
    del A, B, Cd, B_run
    torch.cuda.empty_cache()
    ooc = {}
    if not args.skip_ooc:
        if world == 1:
            # The compat adapter allows one initialisation per process (as the reference's
            # does) and this process used it for the e2e leg: the out-of-core leg runs in a
            # child process on the same GPU while this one waits.
            ooc["compat_c3_form"] = child_c3s(args, local)
        ooc["sharded_c4_form"] = ooc_sharded_leg(args.c4_m, args.c4_n, args.c4_k, 2, 1, world,
                                                 rank, local, dev, barrier, max_over_ranks,
                                                 peak_tflops, h2d, d2h)

    if rank == 0:
        cpu = None
        if world == 1 and not args.skip_cpu_baseline:
            cpu = cpu_baseline_obj(os.cpu_count() or 1)
        line = {
            "metric": METRIC,
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "per_gpu": f"M={M} N={N} K={K}",
                       "parallelism": (f"one {M * world} x {N} x {K} problem split by C rows "
                                       f"over {world} GPUs; each step all-gathers B from "
                                       f"1/{world} column slices over NVLink (NCCL), then "
                                       "the kernel" if world > 1 else "1 GPU"),
                       "l2": "inputs larger than L2 (416 MiB working set per step)",
                       "seeds": "A 10, B 11, C 12 (counter-based uniform[-1,1))"},
            "roofline": {"bound": "fp32", "achieved": achieved, "peak": peak_tflops,
                         "unit": "TFLOP/s", "frac": achieved / peak_tflops, "traffic": traffic,
                         "traffic_source": traffic_source,
                         "kernel_ms": kernel_ms,
                         "peak_source": "measured FP32 pipe probes, this run: the higher of scalar "
                                        "FFMA (xvram_b200_ffma_probe) and packed FFMA2 "
                                        "(xvram_b200_ffma2_probe)",
                         "probes": probes,
                         "peak_nominal_at_sampled_clock":
                             sms * 128 * 2 * (clocks.summary()["sm_mhz"] or 0) * 1e6 / 1e12},
            "host_link": {"h2d_gbs": h2d, "d2h_gbs": d2h, "concurrent_ranks": world,
                          "how": "pinned 256 MiB copies, all ranks at once, min over ranks",
                          "compat_e2e_link_gbs": (h2d_bytes + d2h_bytes) / e2e_s_max / 1e9,
                          "compat_e2e_roofline_ms_serial": 1e3 * t_roof,
                          "compat_e2e_roofline_ms": 1e3 * t_roof_overlap,
                          "compat_e2e_frac_of_roofline": t_roof_overlap / e2e_s_max,
                          "compat_e2e_floor_ms_call_order": 1e3 * t_floor_api,
                          "compat_e2e_frac_of_call_order_floor": t_floor_api / e2e_s_max,
                          "sharded_e2e_link_gbs": (sh_h2d + sh_d2h) / sharded_s / 1e9,
                          "sharded_e2e_roofline_ms": 1e3 * t_roof_sharded,
                          "sharded_e2e_frac_of_roofline": t_roof_sharded / sharded_s},
            "e2e": (
                {"value": FLOP / e2e_s_max / 1e12, "unit": "TFLOP/s",
                 "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                 "ms_per_step": 1e3 * e2e_s_max,
                 "path": "xvram_cuda_compat_get_api: memcpy H2D x3, blas_sgemm, memcpy D2H",
                 "gemm_in_place": int(info.gemm_in_place),
                 "step_ms": {"min": e2e_step_ms[0],
                             "median": e2e_step_ms[len(e2e_step_ms) // 2],
                             "max": e2e_step_ms[-1]},
                 "call_ms_median": e2e_call_ms,
                 "gemm_deferred": int(info.gemm_deferred),
                 "gemm_column_blocks": int(info.gemm_column_blocks),
                 "gemm_streamed": int(info.gemm_streamed),
                 "runtime_h2d_bytes": int(tel.runtime.bytes_h2d)}
                if world == 1 else
                {"value": world * FLOP / sharded_s / 1e12, "unit": "TFLOP/s",
                 "h2d_bytes_per_step": sh_h2d, "d2h_bytes_per_step": sh_d2h,
                 "ms_per_step": 1e3 * sharded_s,
                 "path": "xvram_b200_sgemm_sharded: per rank A rows + 1/N of each B panel H2D, "
                         "NCCL all-gather of B panels over NVLink, C rows H2D/D2H"}),
            "e2e_sharded": {"value": world * FLOP / sharded_s / 1e12, "unit": "TFLOP/s",
                            "ms_per_step": 1e3 * sharded_s, "h2d_bytes_per_step": sh_h2d,
                            "d2h_bytes_per_step": sh_d2h, "panel_k": 1024,
                            "frac_of_roofline": t_roof_sharded / sharded_s,
                            "median_ms": 1e3 * statistics.median(sh_times),
                            "step_ms": [round(1e3 * t, 3) for t in sh_times],
                            "path": "xvram_b200_sgemm_sharded (copies overlap compute)"},
            # per step: the SGEMM kernel plus one transpose per K-major operand (TN: 2)
            "tf32x3": {
                "what": "three-term TF32 on tcgen05/TMEM (math mode 3 / XVRAM_B200_PATH_TF32X3); "
                        "FP32-accurate within max|err|/(K max|a| max|b|) <= 1e-6, not bit-identical",
                "value": world * FLOP / (tc_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": tc_ms,
                "vs_fp32_ffma_peak": FLOP / (tc_ms * 1e-3) / 1e12 / peak_tflops,
                "tensor_pipe": {"bound": "tensor", "tf32_flop_per_step": 3 * FLOP,
                                "achieved_tf32_tflops": 3 * FLOP / (tc_ms * 1e-3) / 1e12,
                                "peak_tf32_tflops": measured_tf32_peak(),
                                "peak_source": "MEASURED_PEAKS.json bf16_tflops / 2 (TF32 runs "
                                               "at half the BF16 tensor rate)",
                                "frac": 3 * FLOP / (tc_ms * 1e-3) / 1e12 / measured_tf32_peak(),
                                "cublas_tf32_tflops_this_run": tf32_cublas,
                                "frac_of_cublas_tf32": 3 * FLOP / (tc_ms * 1e-3) / 1e12
                                                       / tf32_cublas},
                "e2e": {"value": FLOP / e2e_tc_s / 1e12, "unit": "TFLOP/s",
                        "ms_per_step": 1e3 * e2e_tc_s,
                        "step_ms": {"min": tc_step_ms[0],
                                    "median": tc_step_ms[len(tc_step_ms) // 2],
                                    "max": tc_step_ms[-1]},
                        "call_ms_median": tc_call_ms,
                        "path": "compat ABI, blas_set_math_mode(3)"},
                "clocks": tc_clocks.summary(),
            },
            "compat_trace": ({"path": args.trace, "records": trace_records,
                              "format": "xvram.cuda_compat_trace v1 (JSON lines)"}
                             if trace_records is not None else None),
            # the reference's own library contraction on this GPU, same operands, for context
            "library_sgemm": library,
            "ooc": ooc or None,
            "gpu_launches": args.steps * (1 + int(OP_A == 1) + int(OP_B == 0)),
            "gpu_launches_e2e": launches_e2e,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--trace", default=None,
                    help="write one extra compat e2e step as xvram.cuda_compat_trace JSON lines")
    ap.add_argument("--workload", choices=["c2", "c3s", "c4s", "c5"], default="c2",
                    help="c2: the headline (BASELINE config 2); c3s: one out-of-core GEMM; "
                         "c4s: config 4's partitioned form, strong-scaled over the ranks; "
                         "c5: the 24-layer MLP (BASELINE config 5) through the SDK")
    ap.add_argument("--c4-m", type=int, default=65536)
    ap.add_argument("--c4-n", type=int, default=65536)
    ap.add_argument("--c4-k", type=int, default=16384)
    ap.add_argument("--mlp-features", type=int, default=16384)
    ap.add_argument("--mlp-batch", type=int, default=512)
    ap.add_argument("--mlp-layers", type=int, default=24)
    ap.add_argument("--mlp-budget-gib", type=float, default=8.0)
    ap.add_argument("--ooc-n", type=int, default=65536)
    ap.add_argument("--ooc-budget-gib", type=float, default=10.0)
    ap.add_argument("--ooc-tf32-steps", type=int, default=0,
                    help="c3s: calls in math mode 3 (three-term TF32) after the strict ones")
    ap.add_argument("--skip-ooc", action="store_true",
                    help="leave the out-of-core legs (the 'ooc' key) out of the default run")
    args = ap.parse_args()
    if args.warmup < 3 and args.workload == "c2" and args.impl == "ours":
        args.warmup = 3   # the headline line's rule; the single-leg workloads take what is given
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.workload == "c3s":
        run_out_of_core(args)
        return
    if args.workload == "c5":
        run_mlp(args)
        return
    if args.workload == "c4s":
        run_sharded_c4(args)
        return
    main_gpu(args)


if __name__ == "__main__":
    main()
