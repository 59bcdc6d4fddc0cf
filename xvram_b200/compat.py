"""Python view of the cudaMalloc/cudaMemcpy/cublasSgemm-style C table.

``CompatApi`` loads ``xvram_cuda_compat_get_api`` from the native library and calls
the table exactly as a C caller of ``include/xvram_cuda_compat.h`` does (compare the
reference's examples/preview-gemm/main.cpp:18-105): initialise, malloc_device,
memcpy(H2D), blas_create, blas_sgemm, memcpy(D2H), free_device, shutdown.  The
ctypes structures below mirror the C layouts; tests/test_abi_layout.py checks them
against the layout of the reference headers.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

from ._native import lib

u8, u32, u64, i32, i64 = C.c_uint8, C.c_uint32, C.c_uint64, C.c_int32, C.c_int64
f32, f64, vp = C.c_float, C.c_double, C.c_void_p

# Status codes (include/xvram.h)
STATUS_NAMES = [
    "SUCCESS", "INVALID_ARGUMENT", "INCOMPATIBLE_ABI", "UNSUPPORTED", "UNAVAILABLE",
    "HOST_OUT_OF_MEMORY", "DEVICE_OUT_OF_MEMORY", "BUDGET_PRESSURE", "BUSY", "NOT_READY",
    "TIMEOUT", "CORRUPTION", "CALLBACK_FAILED", "CUDA_ERROR", "CUBLAS_ERROR", "POISONED",
    "CLEANUP_FAILED", "CLOSED", "CANCELLED", "INTERNAL",
]
SUCCESS, INVALID_ARGUMENT, INCOMPATIBLE_ABI, UNSUPPORTED = 0, 1, 2, 3
NOT_READY, TIMEOUT, POISONED, CLOSED = 9, 10, 15, 17
H2D, D2H = 1, 2
OP_N, OP_T = 0, 1
STATE_UNINITIALIZED, STATE_INITIALIZING, STATE_READY, STATE_POISONED, STATE_CLOSED = range(5)


class ErrorInfo(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("status", u32), ("native_domain", u32), ("reserved0", u32),
        ("native_code", i64), ("stage", C.c_char * 32), ("operation", C.c_char * 64),
        ("native_name", C.c_char * 64), ("message", C.c_char * 256),
    ]


class SessionConfig(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("flags", u32), ("device_ordinal", i32), ("context_mode", u32),
        ("chunk_size_bytes", u64), ("cache_target_bytes", u64), ("device_headroom_bytes", u64),
        ("workspace_cap_bytes", u64), ("budget_poll_ms", u64), ("max_transaction_ms", u64),
        ("staging_slots", u32), ("cache_policy", u32), ("prefetch_distance", u32),
        ("reserved0", u32), ("reserved", u64 * 4),
    ]


class SessionTelemetry(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("flags", u32), ("cache_target_bytes", u64),
        ("cache_target_minimum_bytes", u64), ("cache_target_maximum_bytes", u64),
        ("resident_bytes", u64), ("resident_bytes_peak", u64), ("workspace_bytes", u64),
        ("bytes_h2d", u64), ("bytes_d2h", u64), ("cache_hits", u64), ("cache_misses", u64),
        ("clean_evictions", u64), ("dirty_evictions", u64), ("writebacks_completed", u64),
        ("mappings", u64), ("unmaps", u64), ("set_access_calls", u64), ("handle_reuses", u64),
        ("unsafe_remaps", u64), ("unsafe_transitions", u64), ("budget_shrinks", u64),
        ("budget_grows", u64), ("cuda_driver_version", u32), ("cublas_version", u32),
        ("cublas_lt_available", u32), ("poisoned", u32), ("physical_handles_created", u64),
        ("physical_handles_released", u64), ("event_boundaries", u64),
        ("pinned_staging_bytes", u64), ("transactions_completed", u64),
        ("algorithm_selections", u64), ("algorithm_cache_hits", u64),
        ("last_transaction_ms", f64), ("budget_sample_count", u64),
        ("cuda_free_bytes_minimum", u64), ("cuda_free_bytes_end", u64),
        ("cublas_lt_version", u32), ("cublas_library_source", u32),
        ("wddm_available_bytes_minimum", u64), ("wddm_available_bytes_end", u64),
        ("wddm_budget_observed", u32), ("watchdog_rejections", u32), ("target_oom_retries", u64),
    ]


class CompatConfig(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("flags", u32), ("session", SessionConfig),
        ("stall_timeout_ms", u64), ("cublas_library", C.c_char * 1024),
        ("cublas_lt_library", C.c_char * 1024), ("reserved", u64 * 4),
    ]


class CompatTelemetry(C.Structure):
    _fields_ = [
        ("struct_size", u32), ("state", u32), ("runtime", SessionTelemetry),
        ("device_ordinal", i32), ("device_count", u32), ("device_name", C.c_char * 128),
        ("total_vram_bytes", u64), ("host_physical_bytes", u64), ("host_available_bytes", u64),
        ("host_store_cap_bytes", u64), ("host_headroom_bytes", u64), ("effective_chunk_bytes", u64),
        ("calls_attempted", u64), ("calls_submitted", u64), ("calls_completed", u64),
        ("calls_rejected", u64), ("allocations_created", u64), ("allocations_released", u64),
        ("live_allocations", u64), ("logical_bytes", u64), ("logical_bytes_peak", u64),
        ("handles_created", u64), ("handles_destroyed", u64), ("live_handles", u64),
        ("h2d_bytes", u64), ("d2h_bytes", u64), ("gemm_calls", u64), ("tiles_submitted", u64),
        ("tiles_retired", u64), ("progress_sequence", u64), ("retired_va_reservations", u64),
        ("retired_va_reservations_freed", u64), ("retired_va_bytes", u64),
        ("retired_va_bytes_freed", u64), ("host_backing_bytes", u64),
        ("host_backing_peak_bytes", u64), ("host_budget_bytes", u64),
        ("cleanup_operations_drained", u32), ("cleanup_events_drained", u32),
        ("cleanup_completed", u32), ("quarantined", u32), ("reserved", u64 * 4),
    ]


_FN = C.CFUNCTYPE
_S = u32  # xvram_status
FN_TYPES = {
    "initialize": _FN(_S, C.POINTER(CompatConfig)),
    "shutdown": _FN(_S),
    "get_error": _FN(_S, C.POINTER(ErrorInfo)),
    "get_telemetry": _FN(_S, C.POINTER(CompatTelemetry)),
    "malloc_device": _FN(_S, C.POINTER(vp), u64),
    "free_device": _FN(_S, vp),
    "memcpy": _FN(_S, vp, vp, u64, u32),
    "get_device": _FN(_S, C.POINTER(i32)),
    "get_device_count": _FN(_S, C.POINTER(i32)),
    "set_device": _FN(_S, i32),
    "synchronize": _FN(_S),
    "mem_get_info": _FN(_S, C.POINTER(u64), C.POINTER(u64)),
    "blas_create": _FN(_S, C.POINTER(vp)),
    "blas_destroy": _FN(_S, vp),
    "blas_get_version": _FN(_S, vp, C.POINTER(i32)),
    "blas_set_stream": _FN(_S, vp, u64),
    "blas_get_stream": _FN(_S, vp, C.POINTER(u64)),
    "blas_set_pointer_mode": _FN(_S, vp, u32),
    "blas_get_pointer_mode": _FN(_S, vp, C.POINTER(u32)),
    "blas_set_math_mode": _FN(_S, vp, u32),
    "blas_get_math_mode": _FN(_S, vp, C.POINTER(u32)),
    "blas_sgemm": _FN(_S, vp, u32, u32, i32, i32, i32, C.POINTER(f32), vp, i32, vp, i32,
                      C.POINTER(f32), vp, i32),
}


class ApiTable(C.Structure):
    _fields_ = ([("struct_size", u32), ("abi_version", u32)] +
                [(name, t) for name, t in FN_TYPES.items()] + [("reserved", u64 * 8)])


def session_config_init() -> SessionConfig:
    """XVRAM_SESSION_CONFIG_V1_INIT."""
    s = SessionConfig()
    s.struct_size = C.sizeof(SessionConfig)
    s.chunk_size_bytes = 64 << 20
    s.device_headroom_bytes = 512 << 20
    s.workspace_cap_bytes = 4 << 20
    s.budget_poll_ms = 100
    s.staging_slots = 4
    s.prefetch_distance = 2
    return s


def compat_config_init() -> CompatConfig:
    """XVRAM_CUDA_COMPAT_CONFIG_V1_INIT."""
    c = CompatConfig()
    c.struct_size = C.sizeof(CompatConfig)
    c.session = session_config_init()
    c.stall_timeout_ms = 5000
    return c


def get_api(version: int = 1, size: Optional[int] = None) -> tuple[int, ApiTable]:
    table = ApiTable()
    st = lib.xvram_cuda_compat_get_api(version, C.sizeof(ApiTable) if size is None else size,
                                       C.byref(table))
    return st, table


class XvramError(RuntimeError):
    def __init__(self, op: str, status: int, info: Optional[ErrorInfo] = None):
        self.op, self.status = op, status
        detail = ""
        if info is not None:
            detail = (f" [{info.stage.decode()}:{info.operation.decode()}] "
                      f"{info.message.decode()} {info.native_name.decode()}")
        name = STATUS_NAMES[status] if status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{op} failed: {name}{detail}")


class CompatApi:
    """The function table with convenience wrappers that raise on failure."""

    def __init__(self):
        st, self.t = get_api()
        if st != SUCCESS:
            raise XvramError("get_api", st)

    # raw table access: api.raw.blas_sgemm(...) returns the status
    @property
    def raw(self) -> ApiTable:
        return self.t

    def error(self) -> ErrorInfo:
        e = ErrorInfo()
        e.struct_size = C.sizeof(ErrorInfo)
        self.t.get_error(C.byref(e))
        return e

    def check(self, op: str, st: int) -> None:
        if st != SUCCESS:
            raise XvramError(op, st, self.error())

    def initialize(self, config: Optional[CompatConfig] = None) -> int:
        cfg = config or compat_config_init()
        return self.t.initialize(C.byref(cfg))

    def shutdown(self) -> int:
        return self.t.shutdown()

    def telemetry(self) -> CompatTelemetry:
        out = CompatTelemetry()
        out.struct_size = C.sizeof(CompatTelemetry)
        self.check("get_telemetry", self.t.get_telemetry(C.byref(out)))
        return out

    def malloc(self, nbytes: int) -> int:
        p = vp()
        self.check("malloc_device", self.t.malloc_device(C.byref(p), nbytes))
        return p.value

    def free(self, ptr: int) -> None:
        self.check("free_device", self.t.free_device(ptr))

    def h2d(self, dst: int, src_ptr: int, nbytes: int) -> None:
        self.check("memcpy(H2D)", self.t.memcpy(dst, src_ptr, nbytes, H2D))

    def d2h(self, dst_ptr: int, src: int, nbytes: int) -> None:
        self.check("memcpy(D2H)", self.t.memcpy(dst_ptr, src, nbytes, D2H))

    def blas_create(self) -> int:
        h = vp()
        self.check("blas_create", self.t.blas_create(C.byref(h)))
        return h.value

    def blas_destroy(self, h: int) -> None:
        self.check("blas_destroy", self.t.blas_destroy(h))

    def sgemm(self, h: int, op_a: int, op_b: int, m: int, n: int, k: int, alpha: float, a: int,
              lda: int, b: int, ldb: int, beta: float, c: int, ldc: int) -> int:
        al, be = f32(alpha), f32(beta)
        return self.t.blas_sgemm(h, op_a, op_b, m, n, k, C.byref(al), a, lda, b, ldb,
                                 C.byref(be), c, ldc)

    def synchronize(self) -> None:
        self.check("synchronize", self.t.synchronize())


def runtime_info() -> "C.Structure":
    from ._native import RuntimeInfo
    out = RuntimeInfo()
    out.struct_size = C.sizeof(RuntimeInfo)
    lib.xvram_b200_compat_runtime_info(C.byref(out))
    return out
