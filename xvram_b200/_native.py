"""ctypes binding of the native library (xvram_b200/lib/libxvram_b200.so).

The library is the product: there is no Python or CPU fallback.  Importing this
module without the built library raises immediately; build it with
``python -m xvram_b200.build`` (``__graft_entry__.build()`` does the same).

``XVRAM_B200_LIBRARY`` in the environment names another build of the same objects to
bind instead; the CPU test suite uses it for its link that also exports the
host-memory fake device seam.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent / "lib"
PRODUCT_LIB_PATH = _LIB_DIR / "libxvram_b200.so"
LIB_PATH = Path(os.environ.get("XVRAM_B200_LIBRARY") or PRODUCT_LIB_PATH)
# The same code linked as the two drop-ins: the compat library exports
# xvram_cuda_compat_get_api only, the SDK library xvram_get_api only.
COMPAT_LIB_PATH = _LIB_DIR / "libxvram_cuda_compat.so"
SDK_LIB_PATH = _LIB_DIR / "libxvram.so"

u32, u64, i32, i64 = C.c_uint32, C.c_uint64, C.c_int32, C.c_int64
f32, f64 = C.c_float, C.c_double
vp = C.c_void_p


class PlanInfo(C.Structure):
    """xvram_b200_plan_info_v1 (include/xvram_b200.h)."""

    _fields_ = [
        ("struct_size", u32), ("status", u32),
        ("block_m", i64), ("block_n", i64), ("panel_k", i64),
        ("n_outer", i32), ("panel_slots", i32), ("c_slots", i32), ("reserved0", i32),
        ("slot_bytes", u64), ("c_slot_bytes", u64),
        ("steps", u64), ("panel_loads", u64), ("panel_hits", u64), ("panel_evictions", u64),
        ("h2d_bytes", u64), ("d2h_bytes", u64),
        ("est_seconds", f64),
    ]


class RuntimeInfo(C.Structure):
    """xvram_b200_runtime_info_v1 (include/xvram_b200.h)."""

    _fields_ = [
        ("struct_size", u32), ("reserved0", u32),
        ("frame_bytes", u64), ("frame_capacity", u64),
        ("gemm_in_place", u64), ("gemm_streamed", u64),
        ("last_block_m", u64), ("last_block_n", u64), ("last_panel_k", u64),
        ("last_steps", u64), ("last_panel_slots", u64),
        ("last_gemm_ms", f64),
        ("gemm_deferred", u64), ("gemm_column_blocks", u64), ("panel_slot_refills", u64),
    ]


class DeviceInfo(C.Structure):
    """xvram_b200_device_info_v1 (include/xvram_b200.h)."""

    _fields_ = [
        ("struct_size", u32), ("ordinal", i32), ("device_count", i32),
        ("name", C.c_char * 128), ("total_bytes", u64), ("free_bytes", u64),
        ("sm_count", i32), ("compute_capability_major", i32), ("compute_capability_minor", i32),
        ("driver_version", i32), ("vmm_granularity", u64), ("runtime_headers_version", i32),
        ("reserved0", i32),
    ]


class ShardCollectives(C.Structure):
    """xvram_b200_shard_collectives_v1 (include/xvram_b200.h)."""

    ALL_REDUCE = C.CFUNCTYPE(u32, vp, C.POINTER(u64), u64, u64)
    ALL_GATHER = C.CFUNCTYPE(u32, vp, C.POINTER(f32), C.POINTER(f32), u64, u64)
    _fields_ = [("struct_size", u32), ("reserved0", u32), ("context", vp),
                ("all_reduce_max_u64", ALL_REDUCE), ("all_gather_f32", ALL_GATHER)]


class ShardPlan(C.Structure):
    """xvram_b200_shard_plan_v1 (include/xvram_b200.h)."""

    _fields_ = [("struct_size", u32), ("world", i32),
                ("m_max", u64), ("avail_min", u64), ("row_groups", u64), ("group_rows", u64),
                ("block_n", u64), ("panel_k", u64), ("b_slice_cols", u64), ("b_slice_k", u64),
                ("slice_elems", u64), ("device_bytes", u64), ("rank", i32), ("reserved0", u32),
                ("gathers", u64), ("h2d_bytes", u64), ("d2h_bytes", u64)]


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with `python -m xvram_b200.build` "
            "(there is no fallback implementation)")
    lib = C.CDLL(str(LIB_PATH))
    lib.xvram_b200_sgemm_device.argtypes = [u32, u32, i64, i64, i64, f32, vp, i64, vp, i64, f32,
                                            vp, i64, u64, u32]
    lib.xvram_b200_sgemm_device.restype = u32
    lib.xvram_b200_sgemm_device_ws.argtypes = [u32, u32, i64, i64, i64, f32, vp, i64, vp, i64,
                                               f32, vp, i64, vp, u64, u64, u32]
    lib.xvram_b200_sgemm_device_ws.restype = u32
    lib.xvram_b200_sgemm_device_noalloc.argtypes = [u32, u32, i64, i64, i64, f32, vp, i64, vp,
                                                    i64, f32, vp, i64, u64, u32]
    lib.xvram_b200_sgemm_device_noalloc.restype = u32
    lib.xvram_b200_sgemm_workspace_bytes.argtypes = [u32, u32, i64, i64, i64]
    lib.xvram_b200_sgemm_workspace_bytes.restype = u64
    lib.xvram_b200_sgemm_tile_shape.argtypes = [i64, i64, C.POINTER(i32), C.POINTER(i32)]
    lib.xvram_b200_sgemm_tile_shape.restype = u32
    lib.xvram_b200_shard_unique_id.argtypes = [vp, u64]
    lib.xvram_b200_shard_unique_id.restype = u32
    lib.xvram_b200_shard_group_create.argtypes = [vp, u64, i32, i32, C.POINTER(u64)]
    lib.xvram_b200_shard_group_create.restype = u32
    lib.xvram_b200_shard_group_create_custom.argtypes = [C.POINTER(ShardCollectives), i32, i32,
                                                         C.POINTER(u64)]
    lib.xvram_b200_shard_group_create_custom.restype = u32
    lib.xvram_b200_shard_rows.argtypes = [i64, i32, i32, C.POINTER(i64), C.POINTER(i64)]
    lib.xvram_b200_shard_rows.restype = u32
    lib.xvram_b200_shard_last_plan.argtypes = [u64, C.POINTER(ShardPlan)]
    lib.xvram_b200_shard_last_plan.restype = u32
    lib.xvram_b200_shard_group_destroy.argtypes = [u64]
    lib.xvram_b200_shard_group_destroy.restype = u32
    lib.xvram_b200_shard_allgather_rows.argtypes = [u64, vp, i64, i64, i64, vp, i64, vp, u64, u64]
    lib.xvram_b200_shard_allgather_rows.restype = u32
    lib.xvram_b200_sgemm_sharded.argtypes = [u64, u32, u32, i64, i64, i64, f32, vp, i64, vp, i64,
                                             f32, vp, i64, i64]
    lib.xvram_b200_sgemm_sharded.restype = u32
    lib.xvram_b200_kernel_status.argtypes = [u64, C.POINTER(u32)]
    lib.xvram_b200_kernel_status.restype = u32
    lib.xvram_b200_fill_uniform.argtypes = [vp, u64, u64, u64, i32]
    lib.xvram_b200_fill_uniform.restype = None
    lib.xvram_b200_plan_panels.argtypes = [u32, u32, i64, i64, i64, i32, u64, u64, f64, f64, f64,
                                           i64, i64, i64, C.POINTER(PlanInfo)]
    lib.xvram_b200_plan_panels.restype = u32
    lib.xvram_b200_plan_steps.argtypes = [u32, u32, i64, i64, i64, i32, u64, u64, i64, i64, i64,
                                          C.POINTER(i32), u64]
    lib.xvram_b200_plan_steps.restype = u32
    arr3 = C.POINTER(u64)
    lib.xvram_b200_validate_gemm.argtypes = [u64, u64, u64, u32, u32, arr3, arr3, arr3, arr3,
                                             arr3, arr3, C.c_char_p]
    lib.xvram_b200_validate_gemm.restype = i32
    lib.xvram_b200_validate_gemm_typed.argtypes = [u64, u64, u64, u32, u32, arr3, arr3, arr3,
                                                   arr3, arr3, arr3, C.POINTER(u32), i32,
                                                   C.c_char_p]
    lib.xvram_b200_validate_gemm_typed.restype = i32
    lib.xvram_b200_gemm_typed_workspace_bytes.argtypes = [u32, u32, i32, u32, u32, i64, i64, i64]
    lib.xvram_b200_gemm_typed_workspace_bytes.restype = u64
    lib.xvram_b200_gemm_device_typed.argtypes = [u32, u32, i32, u32, u32, i64, i64, i64, f64, vp,
                                                 i64, vp, i64, f64, vp, i64, vp, u64, u64]
    lib.xvram_b200_gemm_device_typed.restype = u32
    lib.xvram_b200_ffma_probe.argtypes = [i32, i32, vp, u64]
    lib.xvram_b200_ffma_probe.restype = u32
    lib.xvram_b200_ffma2_probe.argtypes = [i32, i32, vp, u64]
    lib.xvram_b200_ffma2_probe.restype = u32
    lib.xvram_b200_compat_runtime_info.argtypes = [C.POINTER(RuntimeInfo)]
    lib.xvram_b200_compat_runtime_info.restype = u32
    lib.xvram_cuda_compat_get_api.argtypes = [u32, u32, vp]
    lib.xvram_cuda_compat_get_api.restype = u32
    lib.xvram_get_api.argtypes = [u32, u32, vp]
    lib.xvram_get_api.restype = u32
    lib.xvram_b200_bias_activation.argtypes = [u64, i64, i64, i64, u64, u32, u64]
    lib.xvram_b200_bias_activation.restype = u32
    lib.xvram_b200_digest_bench.argtypes = [vp, u64, u64, C.POINTER(u64)]
    lib.xvram_b200_digest_bench.restype = None
    lib.xvram_b200_digest_compat.argtypes = [vp, u64, C.POINTER(u64)]
    lib.xvram_b200_digest_compat.restype = None
    lib.xvram_b200_device_query.argtypes = [i32, C.POINTER(DeviceInfo)]
    lib.xvram_b200_device_query.restype = u32
    if has_test_seam(lib):
        lib.xvram_b200_test_set_device_factory.argtypes = [vp]
        lib.xvram_b200_test_set_device_factory.restype = u32
    return lib


def has_test_seam(handle: C.CDLL) -> bool:
    """True for the test suite's link, which exports the fake-device seam."""
    try:
        handle.xvram_b200_test_set_device_factory
    except AttributeError:
        return False
    return True


lib = _load()

# Every symbol include/*.h declares (checked by tests/test_native_load.py).
EXPORTED = (
    "xvram_cuda_compat_get_api",
    "xvram_get_api",
    "xvram_b200_bias_activation",
    "xvram_b200_device_query",
    "xvram_b200_digest_bench",
    "xvram_b200_digest_compat",
    "xvram_b200_sgemm_device",
    "xvram_b200_sgemm_device_ws",
    "xvram_b200_sgemm_workspace_bytes",
    "xvram_b200_sgemm_tile_shape",
    "xvram_b200_sgemm_device_noalloc",
    "xvram_b200_kernel_status",
    "xvram_b200_shard_unique_id",
    "xvram_b200_shard_group_create",
    "xvram_b200_shard_group_destroy",
    "xvram_b200_shard_group_create_custom",
    "xvram_b200_shard_rows",
    "xvram_b200_shard_last_plan",
    "xvram_b200_shard_allgather_rows",
    "xvram_b200_sgemm_sharded",
    "xvram_b200_fill_uniform",
    "xvram_b200_plan_panels",
    "xvram_b200_plan_steps",
    "xvram_b200_validate_gemm",
    "xvram_b200_validate_gemm_typed",
    "xvram_b200_gemm_typed_workspace_bytes",
    "xvram_b200_gemm_device_typed",
    "xvram_b200_ffma_probe",
    "xvram_b200_ffma2_probe",
    "xvram_b200_compat_runtime_info",
)
