"""Out-of-core SGEMM through the compat table: operands far larger than the device budget,
streamed through the frame pool with eviction and frame reuse, checked against FP64.

Sizes: 32768^3 NT (4 GiB per operand) with a 2.5 GiB budget always; the scaled BASELINE
config 3 (65536^3 NT, beta 1, 16 GiB per operand, 10 GiB budget -- the same budget fraction
as 40 GiB of 192 GiB) when the host has the memory for it.  Each runs in its own process
(one initialisation per process)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent

SCRIPT = r'''
import json, sys, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from oracle_lib import TOLERANCE, load_oracle
from xvram_b200 import compat as cp, device as xd
n, budget_gib = int(sys.argv[2]), float(sys.argv[3])
api = cp.CompatApi()
cfg = cp.compat_config_init()
cfg.session.cache_target_bytes = int(budget_gib * (1 << 30))
api.check("initialize", api.initialize(cfg))
a = np.empty((n, n), np.float32); xd.fill_uniform(a, 100)   # A m x k (op N)
b = np.empty((n, n), np.float32); xd.fill_uniform(b, 101)   # B stored n x k (op T)
c = np.empty((n, n), np.float32); xd.fill_uniform(c, 102)
ptrs = []
for arr in (a, b, c):
    d = api.malloc(arr.nbytes); api.h2d(d, arr.ctypes.data, arr.nbytes); ptrs.append(d)
h = api.blas_create()
api.check("sgemm", api.sgemm(h, 0, 1, n, n, n, 1.0, ptrs[0], n, ptrs[1], n, 1.0, ptrs[2], n))
out = np.empty_like(c)
api.d2h(out.ctypes.data, ptrs[2], out.nbytes)
rng = np.random.default_rng(5)
rows, cols = rng.integers(0, n, 16384), rng.integers(0, n, 16384)
ref = load_oracle().gemm_sampled(0, 1, n, 1.0, a, n, b, n, 1.0, c, n, rows, cols, threads=16)
err = float(np.max(np.abs(out[cols, rows] - ref))) / n
t = api.telemetry(); info = cp.runtime_info()
print(json.dumps(dict(err=err, ok=err <= TOLERANCE, streamed=info.gemm_streamed,
    steps=info.last_steps, block=[info.last_block_m, info.last_block_n, info.last_panel_k],
    refills=info.panel_slot_refills, h2d=t.runtime.bytes_h2d,
    resident_peak=t.runtime.resident_bytes_peak, target=t.runtime.cache_target_bytes,
    tiles=[t.tiles_submitted, t.tiles_retired], gemm_ms=info.last_gemm_ms,
    shutdown=api.shutdown(), maps=api.telemetry().runtime.mappings,
    unmaps=api.telemetry().runtime.unmaps,
    boundaries=api.telemetry().runtime.event_boundaries)))
'''


def host_gib() -> float:
    return os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES") / (1 << 30)


def run(n: int, budget_gib: float, timeout: int) -> dict:
    p = subprocess.run([sys.executable, "-c", SCRIPT, str(HERE.parent), str(n), str(budget_gib)],
                       capture_output=True, text=True, timeout=timeout)
    assert p.returncode == 0, p.stderr[-3000:]
    return json.loads(p.stdout.strip().splitlines()[-1])


def check(r: dict) -> None:
    assert r["ok"], r
    assert r["streamed"] == 1 and r["steps"] > 1
    assert r["refills"] > 0                     # slots of the frame arena reused for new panels
    assert r["maps"] == r["unmaps"] == r["boundaries"] > 0   # every unmap a safe one
    assert r["resident_peak"] <= r["target"]
    assert r["tiles"][0] == r["tiles"][1] == r["steps"]
    assert r["shutdown"] == 0


@pytest.mark.skipif(host_gib() < 40, reason="needs ~30 GiB of host memory")
def test_out_of_core_32768_cubed_2_5_gib_budget():
    check(run(32768, 2.5, 900))


@pytest.mark.skipif(host_gib() < 150, reason="needs ~110 GiB of host memory")
def test_out_of_core_c3_scaled_65536_cubed_10_gib_budget():
    check(run(65536, 10.0, 1800))
