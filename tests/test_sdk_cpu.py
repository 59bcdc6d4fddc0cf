"""SDK v1 table (xvram_get_api) contract checks that need no GPU.

Mirrors the reference's SDK ABI tests (reference tests/unit/sdk_abi_tests.cpp and
tests/contract/sdk_export_contract.py): the table's version handshake, status names,
descriptor validation order and null-handle handling all happen before any device call.
"""
from __future__ import annotations

import ctypes as C

import pytest

from xvram_b200 import sdk
from xvram_b200._native import SDK_LIB_PATH


def table():
    st, t = sdk.get_api()
    assert st == sdk.SUCCESS
    return t


def test_get_api_handshake():
    st, t = sdk.get_api()
    assert st == sdk.SUCCESS
    assert t.struct_size == C.sizeof(sdk.ApiTable) and t.abi_version == 1
    for name in sdk._FN:
        assert getattr(t, name), name
    assert sdk.get_api(version=2)[0] == sdk.INCOMPATIBLE_ABI
    assert sdk.get_api(version=0)[0] == sdk.INCOMPATIBLE_ABI
    assert sdk.get_api(size=C.sizeof(sdk.ApiTable) - 8)[0] == sdk.INVALID_ARGUMENT
    from xvram_b200._native import lib
    assert lib.xvram_get_api(1, C.sizeof(sdk.ApiTable), None) == sdk.INVALID_ARGUMENT


def test_sdk_drop_in_library_serves_the_same_table():
    drop_in = C.CDLL(str(SDK_LIB_PATH))
    st, t = sdk.get_api(library=drop_in)
    assert st == sdk.SUCCESS and t.abi_version == 1
    assert t.status_name(sdk.BUDGET_PRESSURE) == b"budget_pressure"


def test_status_names():
    t = table()
    names = ["success", "invalid_argument", "incompatible_abi", "unsupported", "unavailable",
             "host_out_of_memory", "device_out_of_memory", "budget_pressure", "busy", "not_ready",
             "timeout", "corruption", "callback_failed", "cuda_error", "cublas_error", "poisoned",
             "cleanup_failed", "closed", "cancelled", "internal"]
    for code, name in enumerate(names):
        assert t.status_name(code) == name.encode()
    assert t.status_name(99) == b"unknown"


@pytest.mark.parametrize("field,value,status", [
    ("struct_size", 8, sdk.INCOMPATIBLE_ABI),
    ("flags", 1, sdk.INVALID_ARGUMENT),
    ("reserved0", 1, sdk.INVALID_ARGUMENT),
    ("context_mode", 2, sdk.INVALID_ARGUMENT),
    ("cache_policy", 2, sdk.INVALID_ARGUMENT),
    ("device_ordinal", -1, sdk.INVALID_ARGUMENT),
    ("chunk_size_bytes", 0, sdk.INVALID_ARGUMENT),
    ("staging_slots", 1, sdk.INVALID_ARGUMENT),
    ("staging_slots", 9, sdk.INVALID_ARGUMENT),
    ("prefetch_distance", 9, sdk.INVALID_ARGUMENT),
    ("budget_poll_ms", 0, sdk.INVALID_ARGUMENT),
    ("max_transaction_ms", 1 << 63, sdk.INVALID_ARGUMENT),
    ("context_mode", 1, sdk.UNSUPPORTED),
])
def test_session_config_rejected_before_any_device_call(field, value, status):
    t = table()
    cfg = sdk.session_config(**{field: value})
    out = C.c_void_p(1234)
    assert t.session_create(C.byref(cfg), C.byref(out)) == status
    assert out.value is None


def test_session_create_null_arguments():
    t = table()
    cfg = sdk.session_config()
    assert t.session_create(C.byref(cfg), None) == sdk.INVALID_ARGUMENT
    out = C.c_void_p()
    assert t.session_create(None, C.byref(out)) == sdk.INCOMPATIBLE_ABI
    cfg.reserved[2] = 7
    assert t.session_create(C.byref(cfg), C.byref(out)) == sdk.INVALID_ARGUMENT


def test_null_handles_are_invalid_arguments():
    t = table()
    info = sdk.OperationInfo(struct_size=C.sizeof(sdk.OperationInfo))
    err = sdk.ErrorInfo(struct_size=C.sizeof(sdk.ErrorInfo))
    tel = sdk.Telemetry(struct_size=C.sizeof(sdk.Telemetry))
    pinfo = sdk.PlanInfo(struct_size=C.sizeof(sdk.PlanInfo))
    ainfo = sdk.AllocationInfo(struct_size=C.sizeof(sdk.AllocationInfo))
    out = C.c_void_p()
    buf = (C.c_char * 16)()
    assert t.session_get_error(None, C.byref(err)) == sdk.INVALID_ARGUMENT
    assert t.session_get_telemetry(None, C.byref(tel)) == sdk.INVALID_ARGUMENT
    assert t.session_drain(None, 0) == sdk.INVALID_ARGUMENT
    assert t.session_close(None, 0) == sdk.INVALID_ARGUMENT
    t.session_release(None)
    d = sdk.AllocationDesc(struct_size=C.sizeof(sdk.AllocationDesc), size_bytes=64)
    assert t.allocation_create(None, C.byref(d), C.byref(out)) == sdk.INVALID_ARGUMENT
    assert t.allocation_create(None, C.byref(d), None) == sdk.INVALID_ARGUMENT
    assert t.allocation_get_info(None, C.byref(ainfo)) == sdk.INVALID_ARGUMENT
    assert t.allocation_write(None, 0, buf, 16) == sdk.INVALID_ARGUMENT
    assert t.allocation_read(None, 0, buf, 16) == sdk.INVALID_ARGUMENT
    assert t.allocation_release(None) == sdk.INVALID_ARGUMENT
    assert t.prefetch_submit(None, None, C.byref(out)) == sdk.INVALID_ARGUMENT
    assert t.transaction_submit(None, None, C.byref(out)) == sdk.INVALID_ARGUMENT
    assert t.transaction_execute(None, None, 0) == sdk.INVALID_ARGUMENT
    assert t.gemm_plan_create(None, None, C.byref(out)) == sdk.INVALID_ARGUMENT
    assert t.gemm_plan_get_info(None, C.byref(pinfo)) == sdk.INVALID_ARGUMENT
    assert t.gemm_submit(None, C.byref(out)) == sdk.INVALID_ARGUMENT
    assert t.gemm_execute(None, 0) == sdk.INVALID_ARGUMENT
    t.gemm_plan_release(None)
    assert t.operation_poll(None, C.byref(info)) == sdk.INVALID_ARGUMENT
    assert t.operation_wait(None, 0, C.byref(info)) == sdk.INVALID_ARGUMENT
    assert t.operation_cancel(None) == sdk.INVALID_ARGUMENT
    assert t.operation_get_error(None, C.byref(err)) == sdk.INVALID_ARGUMENT
    t.operation_release(None)


def test_session_without_a_device_fails_cleanly():
    """On a machine without a GPU the worker thread's runtime open fails; the call
    returns that failure and leaves nothing running."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    t = table()
    cfg = sdk.session_config()
    out = C.c_void_p()
    st = t.session_create(C.byref(cfg), C.byref(out))
    assert st in (sdk.CUDA_ERROR, sdk.UNAVAILABLE, sdk.DEVICE_OUT_OF_MEMORY)
    assert out.value is None
