"""ctypes binding of the SDK v1 table (include/xvram.h: xvram_get_api).

Mirrors the reference SDK's C interface (reference include/xvram/xvram.h:152-533) one
structure and one function pointer at a time, so tests and scripts drive exactly what a
C caller would.  ``Sdk`` wraps the table with small conveniences (status checks, matrix
descriptors, transaction callbacks); every call still goes through the C ABI.
"""
from __future__ import annotations

import ctypes as C

from ._native import lib

u32, u64, i32, i64, f64 = C.c_uint32, C.c_uint64, C.c_int32, C.c_int64, C.c_double
vp = C.c_void_p
TIMEOUT_INFINITE = (1 << 64) - 1

# status codes (include/xvram/xvram.h)
(SUCCESS, INVALID_ARGUMENT, INCOMPATIBLE_ABI, UNSUPPORTED, UNAVAILABLE, HOST_OUT_OF_MEMORY,
 DEVICE_OUT_OF_MEMORY, BUDGET_PRESSURE, BUSY, NOT_READY, TIMEOUT, CORRUPTION, CALLBACK_FAILED,
 CUDA_ERROR, CUBLAS_ERROR, POISONED, CLEANUP_FAILED, CLOSED, CANCELLED, INTERNAL) = range(20)
QUEUED, RUNNING, COMPLETED, OP_CANCELLED, FAILED = range(5)
READ, READ_WRITE, WRITE_ONLY = range(3)
FP16, BF16, FP32, FP64 = range(4)
COMPUTE_AUTO, COMPUTE_FP32_STRICT, COMPUTE_FP32_TF32, COMPUTE_FP64 = range(4)
ROW_MAJOR, COLUMN_MAJOR = 0, 1
OP_N, OP_T = 0, 1
CACHE_POLICY_CLOCK, CACHE_POLICY_LRU = 0, 1
ZERO_INITIALIZE = 1


class ErrorInfo(C.Structure):
    _fields_ = [("struct_size", u32), ("status", u32), ("native_domain", u32), ("reserved0", u32),
                ("native_code", i64), ("stage", C.c_char * 32), ("operation", C.c_char * 64),
                ("native_name", C.c_char * 64), ("message", C.c_char * 256)]


class SessionConfig(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("device_ordinal", i32),
                ("context_mode", u32), ("chunk_size_bytes", u64), ("cache_target_bytes", u64),
                ("device_headroom_bytes", u64), ("workspace_cap_bytes", u64),
                ("budget_poll_ms", u64), ("max_transaction_ms", u64), ("staging_slots", u32),
                ("cache_policy", u32), ("prefetch_distance", u32), ("reserved0", u32),
                ("reserved", u64 * 4)]


class Telemetry(C.Structure):
    _fields_ = [(n, u64) for n in (
        "cache_target_bytes", "cache_target_minimum_bytes", "cache_target_maximum_bytes",
        "resident_bytes", "resident_bytes_peak", "workspace_bytes", "bytes_h2d", "bytes_d2h",
        "cache_hits", "cache_misses", "clean_evictions", "dirty_evictions", "writebacks_completed",
        "mappings", "unmaps", "set_access_calls", "handle_reuses", "unsafe_remaps",
        "unsafe_transitions", "budget_shrinks", "budget_grows")]
    _fields_ = [("struct_size", u32), ("flags", u32)] + _fields_ + [
        ("cuda_driver_version", u32), ("cublas_version", u32), ("cublas_lt_available", u32),
        ("poisoned", u32), ("physical_handles_created", u64), ("physical_handles_released", u64),
        ("event_boundaries", u64), ("pinned_staging_bytes", u64), ("transactions_completed", u64),
        ("algorithm_selections", u64), ("algorithm_cache_hits", u64),
        ("last_transaction_ms", f64), ("budget_sample_count", u64),
        ("cuda_free_bytes_minimum", u64), ("cuda_free_bytes_end", u64),
        ("cublas_lt_version", u32), ("cublas_library_source", u32),
        ("wddm_available_bytes_minimum", u64), ("wddm_available_bytes_end", u64),
        ("wddm_budget_observed", u32), ("watchdog_rejections", u32), ("target_oom_retries", u64)]


class AllocationDesc(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("size_bytes", u64),
                ("alignment_bytes", u64), ("priority", u32), ("reserved0", u32),
                ("reserved", u64 * 2)]


class AllocationInfo(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("allocation_id", u64),
                ("size_bytes", u64), ("alignment_bytes", u64), ("priority", u32),
                ("stable_virtual_address", u32), ("reserved", u64 * 2)]


class AccessRange(C.Structure):
    _fields_ = [("allocation", vp), ("offset_bytes", u64), ("length_bytes", u64), ("mode", u32),
                ("reserved0", u32)]


class PrefetchDesc(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("ranges", C.POINTER(AccessRange)),
                ("range_count", u64), ("deadline_ms", u64), ("reserved", u64 * 2)]


class ResolvedRange(C.Structure):
    _fields_ = [("allocation_id", u64), ("offset_bytes", u64), ("length_bytes", u64),
                ("device_address", u64), ("mode", u32), ("reserved0", u32)]


class TransactionContext(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("operation_id", u64),
                ("transaction_id", u64), ("ranges", C.POINTER(ResolvedRange)),
                ("range_count", u64), ("workspace_device_address", u64),
                ("workspace_bytes", u64), ("native_stream", u64), ("reserved", u64 * 2)]


TransactionCallback = C.CFUNCTYPE(u32, C.POINTER(TransactionContext), vp, C.POINTER(ErrorInfo))


class TransactionDesc(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("ranges", C.POINTER(AccessRange)),
                ("range_count", u64), ("workspace_bytes", u64), ("deadline_ms", u64),
                ("callback", TransactionCallback), ("user_data", vp), ("reserved", u64 * 2)]


class OperationInfo(C.Structure):
    _fields_ = [("struct_size", u32), ("state", u32), ("result", u32), ("reserved0", u32),
                ("operation_id", u64), ("units_completed", u64), ("units_total", u64),
                ("elapsed_ms", f64), ("bytes_h2d", u64), ("bytes_d2h", u64),
                ("cache_hits", u64), ("cache_misses", u64), ("reserved", u64 * 2)]


class Matrix(C.Structure):
    _fields_ = [("struct_size", u32), ("data_type", u32), ("allocation", vp),
                ("offset_bytes", u64), ("rows", u64), ("columns", u64),
                ("leading_dimension", u64), ("layout", u32), ("reserved0", u32),
                ("reserved", u64 * 2)]


class GemmDesc(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("a", Matrix), ("b", Matrix),
                ("c", Matrix), ("operation_a", u32), ("operation_b", u32),
                ("compute_mode", u32), ("reserved0", u32), ("alpha", f64), ("beta", f64),
                ("workspace_cap_bytes", u64), ("deadline_ms", u64), ("tile_m_hint", u64),
                ("tile_n_hint", u64), ("tile_k_hint", u64), ("reserved", u64 * 3)]


class PlanInfo(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("m", u64), ("n", u64), ("k", u64),
                ("tile_m", u64), ("tile_n", u64), ("tile_k", u64),
                ("maximum_working_set_bytes", u64), ("workspace_bytes", u64),
                ("tile_count", u64), ("effective_compute_mode", u32), ("uses_cublas_lt", u32),
                ("reserved", u64 * 2)]


_FN = {
    "status_name": C.CFUNCTYPE(C.c_char_p, u32),
    "session_create": C.CFUNCTYPE(u32, C.POINTER(SessionConfig), C.POINTER(vp)),
    "session_get_error": C.CFUNCTYPE(u32, vp, C.POINTER(ErrorInfo)),
    "session_get_telemetry": C.CFUNCTYPE(u32, vp, C.POINTER(Telemetry)),
    "session_drain": C.CFUNCTYPE(u32, vp, u64),
    "session_close": C.CFUNCTYPE(u32, vp, u64),
    "session_release": C.CFUNCTYPE(None, vp),
    "allocation_create": C.CFUNCTYPE(u32, vp, C.POINTER(AllocationDesc), C.POINTER(vp)),
    "allocation_get_info": C.CFUNCTYPE(u32, vp, C.POINTER(AllocationInfo)),
    "allocation_write": C.CFUNCTYPE(u32, vp, u64, vp, u64),
    "allocation_read": C.CFUNCTYPE(u32, vp, u64, vp, u64),
    "allocation_release": C.CFUNCTYPE(u32, vp),
    "prefetch_submit": C.CFUNCTYPE(u32, vp, C.POINTER(PrefetchDesc), C.POINTER(vp)),
    "transaction_submit": C.CFUNCTYPE(u32, vp, C.POINTER(TransactionDesc), C.POINTER(vp)),
    "transaction_execute": C.CFUNCTYPE(u32, vp, C.POINTER(TransactionDesc), u64),
    "gemm_plan_create": C.CFUNCTYPE(u32, vp, C.POINTER(GemmDesc), C.POINTER(vp)),
    "gemm_plan_get_info": C.CFUNCTYPE(u32, vp, C.POINTER(PlanInfo)),
    "gemm_submit": C.CFUNCTYPE(u32, vp, C.POINTER(vp)),
    "gemm_execute": C.CFUNCTYPE(u32, vp, u64),
    "gemm_plan_release": C.CFUNCTYPE(None, vp),
    "operation_poll": C.CFUNCTYPE(u32, vp, C.POINTER(OperationInfo)),
    "operation_wait": C.CFUNCTYPE(u32, vp, u64, C.POINTER(OperationInfo)),
    "operation_cancel": C.CFUNCTYPE(u32, vp),
    "operation_get_error": C.CFUNCTYPE(u32, vp, C.POINTER(ErrorInfo)),
    "operation_release": C.CFUNCTYPE(None, vp),
}


class ApiTable(C.Structure):
    _fields_ = ([("struct_size", u32), ("abi_version", u32)] +
                [(name, fn) for name, fn in _FN.items()] + [("reserved", u64 * 16)])


def get_api(version: int = 1, size: int | None = None, library=None):
    table = ApiTable()
    lib_ = library or lib
    lib_.xvram_get_api.argtypes = [u32, u32, vp]
    lib_.xvram_get_api.restype = u32
    st = lib_.xvram_get_api(version, C.sizeof(table) if size is None else size, C.byref(table))
    return st, table


def session_config(**kw) -> SessionConfig:
    """XVRAM_SESSION_CONFIG_V1_INIT with overrides."""
    c = SessionConfig(struct_size=C.sizeof(SessionConfig), chunk_size_bytes=64 << 20,
                      device_headroom_bytes=512 << 20, workspace_cap_bytes=4 << 20,
                      budget_poll_ms=100, staging_slots=4, prefetch_distance=2)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def matrix(alloc, rows: int, cols: int, ld: int, layout: int = COLUMN_MAJOR, offset: int = 0,
           data_type: int = FP32) -> Matrix:
    return Matrix(struct_size=C.sizeof(Matrix), data_type=data_type,
                  allocation=alloc.handle if hasattr(alloc, "handle") else alloc,
                  offset_bytes=offset, rows=rows, columns=cols, leading_dimension=ld,
                  layout=layout)


class SdkError(RuntimeError):
    def __init__(self, what: str, status: int, info: ErrorInfo | None = None):
        detail = ""
        if info is not None:
            detail = (f" [{info.stage.decode()}/{info.operation.decode()}: "
                      f"{info.message.decode()}]")
        super().__init__(f"{what} failed with status {status}{detail}")
        self.status = status


class Allocation:
    def __init__(self, sdk: "Sdk", handle: int, size: int):
        self.sdk, self.handle, self.size = sdk, handle, size

    def write(self, src, offset: int = 0, nbytes: int | None = None) -> None:
        ptr, n = _buf(src)
        self.sdk.check("allocation_write",
                       self.sdk.t.allocation_write(self.handle, offset, ptr, n if nbytes is None else nbytes))

    def read(self, dst, offset: int = 0, nbytes: int | None = None) -> None:
        ptr, n = _buf(dst)
        self.sdk.check("allocation_read",
                       self.sdk.t.allocation_read(self.handle, offset, ptr, n if nbytes is None else nbytes))

    def info(self) -> AllocationInfo:
        out = AllocationInfo(struct_size=C.sizeof(AllocationInfo))
        self.sdk.check("allocation_get_info",
                       self.sdk.t.allocation_get_info(self.handle, C.byref(out)))
        return out

    def release(self) -> int:
        st = self.sdk.t.allocation_release(self.handle)
        if st == SUCCESS:
            self.handle = None
        return st


def _buf(x):
    if hasattr(x, "data_ptr"):
        return x.data_ptr(), x.numel() * x.element_size()
    return x.ctypes.data, x.nbytes


class Sdk:
    """One session of the SDK table (closing it on exit)."""

    def __init__(self, config: SessionConfig | None = None, library=None):
        st, self.t = get_api(library=library)
        if st != SUCCESS:
            raise SdkError("xvram_get_api", st)
        self.cfg = config or session_config()
        self.session = vp()
        st = self.t.session_create(C.byref(self.cfg), C.byref(self.session))
        if st != SUCCESS:
            raise SdkError("session_create", st)
        self._callbacks = []  # keep ctypes callbacks alive while the session may call them

    def error(self) -> ErrorInfo:
        info = ErrorInfo(struct_size=C.sizeof(ErrorInfo))
        self.t.session_get_error(self.session, C.byref(info))
        return info

    def check(self, what: str, st: int) -> None:
        if st != SUCCESS:
            raise SdkError(what, st, self.error())

    def telemetry(self) -> Telemetry:
        t = Telemetry(struct_size=C.sizeof(Telemetry))
        self.check("session_get_telemetry", self.t.session_get_telemetry(self.session, C.byref(t)))
        return t

    def alloc(self, size: int, zero: bool = False, alignment: int = 0) -> Allocation:
        d = AllocationDesc(struct_size=C.sizeof(AllocationDesc), size_bytes=size,
                           flags=ZERO_INITIALIZE if zero else 0, alignment_bytes=alignment)
        h = vp()
        self.check("allocation_create", self.t.allocation_create(self.session, C.byref(d), C.byref(h)))
        return Allocation(self, h.value, size)

    def gemm_desc(self, a: Matrix, b: Matrix, c: Matrix, op_a=OP_N, op_b=OP_N, alpha=1.0,
                  beta=0.0, mode=COMPUTE_AUTO, deadline_ms=0) -> GemmDesc:
        return GemmDesc(struct_size=C.sizeof(GemmDesc), a=a, b=b, c=c, operation_a=op_a,
                        operation_b=op_b, compute_mode=mode, alpha=alpha, beta=beta,
                        deadline_ms=deadline_ms)

    def plan(self, desc: GemmDesc) -> int:
        h = vp()
        self.check("gemm_plan_create", self.t.gemm_plan_create(self.session, C.byref(desc), C.byref(h)))
        return h.value

    def try_plan(self, desc: GemmDesc) -> tuple[int, int]:
        """gemm_plan_create without raising: (status, plan handle or 0)."""
        h = vp()
        st = self.t.gemm_plan_create(self.session, C.byref(desc), C.byref(h))
        return st, (h.value or 0)

    def plan_info(self, plan: int) -> PlanInfo:
        info = PlanInfo(struct_size=C.sizeof(PlanInfo))
        self.check("gemm_plan_get_info", self.t.gemm_plan_get_info(plan, C.byref(info)))
        return info

    def ranges(self, spec) -> C.Array:
        arr = (AccessRange * len(spec))()
        for i, (alloc, off, length, mode) in enumerate(spec):
            arr[i] = AccessRange(allocation=alloc.handle, offset_bytes=off, length_bytes=length,
                                 mode=mode)
        return arr

    def transaction_desc(self, spec, fn, workspace_bytes=0, deadline_ms=0):
        """fn(context) -> status; spec = [(allocation, offset, length, mode), ...]."""
        def trampoline(ctx, _user, _err):
            try:
                return int(fn(ctx.contents))
            except Exception:  # a Python exception must not unwind into C
                return CALLBACK_FAILED
        cb = TransactionCallback(trampoline)
        self._callbacks.append(cb)
        arr = self.ranges(spec)
        d = TransactionDesc(struct_size=C.sizeof(TransactionDesc),
                            ranges=C.cast(arr, C.POINTER(AccessRange)), range_count=len(spec),
                            workspace_bytes=workspace_bytes, deadline_ms=deadline_ms, callback=cb)
        d._keep = arr
        return d

    def prefetch_desc(self, spec, deadline_ms=0) -> PrefetchDesc:
        arr = self.ranges(spec)
        d = PrefetchDesc(struct_size=C.sizeof(PrefetchDesc),
                         ranges=C.cast(arr, C.POINTER(AccessRange)), range_count=len(spec),
                         deadline_ms=deadline_ms)
        d._keep = arr
        return d

    def wait(self, op: int, timeout_ms: int = TIMEOUT_INFINITE) -> OperationInfo:
        info = OperationInfo(struct_size=C.sizeof(OperationInfo))
        self.check("operation_wait", self.t.operation_wait(op, timeout_ms, C.byref(info)))
        return info

    def op_error(self, op: int) -> ErrorInfo:
        info = ErrorInfo(struct_size=C.sizeof(ErrorInfo))
        self.t.operation_get_error(op, C.byref(info))
        return info

    def close(self) -> None:
        if self.session:
            self.t.session_close(self.session, TIMEOUT_INFINITE)
            self.t.session_release(self.session)
            self.session = vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def bias_activation(y_addr: int, ldy: int, rows: int, cols: int, bias_addr: int, relu: bool,
                    stream: int) -> int:
    """xvram_b200_bias_activation: for use inside transaction callbacks."""
    return lib.xvram_b200_bias_activation(y_addr, ldy, rows, cols, bias_addr, 1 if relu else 0,
                                          stream)
