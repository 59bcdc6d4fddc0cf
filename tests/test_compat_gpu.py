"""The compat C table end to end on the GPU (each scenario in a fresh process)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
S = {"SUCCESS": 0, "INVALID_ARGUMENT": 1, "UNSUPPORTED": 3, "NOT_READY": 9, "CLOSED": 17}


def run(name: str, timeout: int = 600) -> dict:
    p = subprocess.run([sys.executable, str(HERE / "compat_scenarios.py"), name],
                       capture_output=True, text=True, timeout=timeout)
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
    assert r["clean_evictions"] > 0 and r["handle_reuses"] > 0
    assert r["dirty_evictions"] > 0           # the device-resident A/B written back first
    assert r["resident_peak"] <= r["cache_target"]
    assert r["mappings_end"] == r["unmaps_end"]
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
