"""The compat C table end to end on the GPU (each scenario in a fresh process)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
S = {"SUCCESS": 0, "INVALID_ARGUMENT": 1, "UNSUPPORTED": 3, "NOT_READY": 9, "CLOSED": 17}


def run(name: str, timeout: int = 600, env: dict | None = None) -> dict:
    p = subprocess.run([sys.executable, str(HERE / "compat_scenarios.py"), name],
                       capture_output=True, text=True, timeout=timeout, env=env)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    return json.loads(p.stdout.strip().splitlines()[-1])


def test_preview_flow():
    r = run("preview")
    assert r["ok"] and r["gemm_calls"] == 1
    assert r["live_allocations"] == 0 and r["live_handles"] == 0
    assert r["shutdown"] == 0 and r["state"] == 4 and r["cleanup_completed"] == 1


def test_padded_suite_all_operations():
    r = run("padded")
    assert r.pop("shutdown") == 0
    assert all(r.values()), r


def test_error_classes():
    r = run("errors")
    assert r["before_init"] == S["NOT_READY"]
    assert r["bad_config"] == S["INVALID_ARGUMENT"] and r["bad_chunk"] == S["INVALID_ARGUMENT"]
    assert r["ok"] == 0
    for key in ("ld_small", "alias", "foreign", "misaligned", "oob", "bad_handle", "free_interior",
                "memcpy_oob", "memcpy_host_is_managed", "double_free", "use_after_free"):
        assert r[key] == S["INVALID_ARGUMENT"], key
    for key in ("bad_op", "zero_m", "nan_alpha", "set_device_other", "set_stream",
                "pointer_mode_device", "math_tensor_op", "memcpy_d2d"):
        assert r[key] == S["UNSUPPORTED"], key
    assert r["math_tf32"] == 0 and r["math_pedantic"] == 0
    assert r["free_null"] == 0 and r["free"] == 0
    assert r["shutdown"] == 0 and r["after_shutdown"] == S["CLOSED"]
    assert r["second_init"] == S["CLOSED"] and r["state"] == 4 and r["attempted_eq"]


def test_out_of_core_eviction_and_reuse():
    r = run("out_of_core")
    assert r["ok"], r
    assert r["streamed"] == 2 and r["in_place"] == 0
    assert r["tiles_submitted"] == r["tiles_retired"] > 2
    # the reference's counters: evictions and handle reuses are VMM unmaps and remaps
    assert r["dirty_evictions"] > 0           # the device-resident A/B written back first
    assert r["handle_reuses"] > 0             # the second streamed GEMM remaps used frames
    assert r["panel_slot_refills"] > 0        # panels replaced in mapped slots (own counter)
    assert r["resident_peak"] <= r["cache_target"]
    assert r["mappings_end"] == r["unmaps_end"] == r["event_boundaries_end"]
    assert r["shutdown"] == 0


def test_in_place_two_passes():
    r = run("in_place_two_passes")
    assert r["ok"], r
    assert r["in_place"] == 2 and r["streamed"] == 0


def test_tensor_core_math_mode_in_place_and_streamed():
    r = run("tensor_cores")
    assert r["mode"] == 3
    assert r["ok"], r
    assert r["in_place_calls"] == 1 and r["streamed_calls"] == 1
    assert r["shutdown"] == 0


def test_deferred_column_blocks_bit_identical_to_synchronous():
    """The default blas_sgemm returns before its kernels finish and runs C as column
    blocks; its results equal the reference's synchronous completion
    (XVRAM_B200_SYNC_GEMM=1) bit for bit, for every operation in strict FP32 and in TF32
    tensor-op math, with ldc > m and reads of C that cut through blocks."""
    env = {k: v for k, v in os.environ.items() if k != "XVRAM_B200_SYNC_GEMM"}
    d = run("deferred", env=env)
    s = run("deferred", env=dict(env, XVRAM_B200_SYNC_GEMM="1"))
    # strict: 64 x 16 tiles of 128 x 256 on 148 SMs; TF32: 32 x 16 tiles of 256 x 256 on
    # 74 SM pairs; 6 blocks of 768 columns (the last 256) either way
    assert d["in_place"] == 8 and d["deferred"] == 8 and d["blocks"] == 8 * 6
    assert s["deferred"] == 0 and s["blocks"] == 0
    assert d["digests"] == s["digests"]
    assert max(d["errors"].values()) <= 1e-6 and d["pad_kept"]
    assert d["shutdown"] == 0 and s["shutdown"] == 0


def test_deferred_result_survives_eviction():
    """A deferred GEMM's unread C is written back to the host when a streamed GEMM needs
    its frames; the values read afterwards, and after a second deferred update, are right."""
    r = run("deferred_evict")
    assert r["streamed"] == 1 and r["dirty_evictions"] > 0
    assert r["deferred"] == 2 and r["blocks"] == 2 * 6
    assert r["evicted_err"] <= 1e-6 and r["second_err"] <= 1e-6
    assert r["shutdown"] == 0
