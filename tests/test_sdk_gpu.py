"""SDK v1 (xvram_get_api) on the GPU: allocations, GEMM plans, transactions, prefetch and
the operation lifecycle, checked against the FP64 oracle / numpy.

Follows the reference's SDK behaviour (reference src/sdk/api.cpp, src/sdk/runtime.cpp):
operations run in submission order on the session worker, queued operations can be
cancelled, running ones answer BUSY, deadlines count from submission.
"""
from __future__ import annotations

import ctypes as C
import threading
import time

import numpy as np
import pytest

from oracle_lib import TOLERANCE, load_oracle, normalized_error

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import sdk  # noqa: E402

MiB = 1 << 20


@pytest.fixture()
def s():
    with sdk.Sdk(sdk.session_config()) as session:
        yield session


def upload(s, arr):
    a = s.alloc(arr.nbytes)
    a.write(np.ascontiguousarray(arr))
    return a


def download(alloc, shape, dtype=np.float32):
    out = np.empty(shape, dtype=dtype)
    alloc.read(out)
    return out


def test_allocation_round_trip_and_zero_initialize(s):
    data = np.arange(1 << 20, dtype=np.float32)
    a = upload(s, data)
    assert np.array_equal(download(a, data.shape), data)
    part = np.full(100, 7.0, dtype=np.float32)
    a.write(part, offset=4 * 1000)
    back = download(a, data.shape)
    assert np.all(back[1000:1100] == 7.0) and back[999] == 999.0 and back[1100] == 1100.0
    z = s.alloc(3 * MiB + 12, zero=True)
    assert not np.any(download(z, (3 * MiB + 12) // 4))
    info = sdk.AllocationInfo(struct_size=C.sizeof(sdk.AllocationInfo))
    s.check("get_info", s.t.allocation_get_info(z.handle, C.byref(info)))
    assert info.size_bytes == 3 * MiB + 12 and info.flags == sdk.ZERO_INITIALIZE
    assert info.stable_virtual_address == 1
    # out-of-range access is an argument error, not a partial copy
    buf = np.zeros(4, dtype=np.float32)
    assert s.t.allocation_read(z.handle, 3 * MiB + 8, buf.ctypes.data, 16) == sdk.INVALID_ARGUMENT
    assert z.release() == sdk.SUCCESS and a.release() == sdk.SUCCESS


@pytest.mark.parametrize("mode", [sdk.COMPUTE_FP32_STRICT, sdk.COMPUTE_AUTO])
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_column_major_gemm_matches_oracle(s, op_a, op_b, mode):
    """Strict FP32, and AUTO, which on FP32 data selects TF32 as in the reference (here the
    FP32-accurate three-term kernel)."""
    orc = load_oracle()
    m, n, k = 515, 389, 611
    a = orc.uniform(m * k, 21)
    b = orc.uniform(k * n, 22)
    c = orc.uniform(m * n, 23)
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    A, B, Cm = upload(s, a), upload(s, b), upload(s, c)
    desc = s.gemm_desc(sdk.matrix(A, m if op_a == 0 else k, k if op_a == 0 else m, lda),
                       sdk.matrix(B, k if op_b == 0 else n, n if op_b == 0 else k, ldb),
                       sdk.matrix(Cm, m, n, m), op_a, op_b, alpha=0.75, beta=-1.25, mode=mode)
    plan = s.plan(desc)
    info = s.plan_info(plan)
    assert (info.m, info.n, info.k, info.tile_count) == (m, n, k, 1)
    want = sdk.COMPUTE_FP32_STRICT if mode == sdk.COMPUTE_FP32_STRICT else sdk.COMPUTE_FP32_TF32
    assert info.effective_compute_mode == want and info.uses_cublas_lt == 0
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    out = download(Cm, (n, m))
    ref = orc.gemm(op_a, op_b, m, n, k, 0.75, a, lda, b, ldb, -1.25, c, m)
    assert normalized_error(out, ref, k, 1.0, 1.0) <= TOLERANCE


@pytest.mark.parametrize("layouts", ["RRR", "RCR", "CRC", "CCR"])
def test_row_major_layouts(s, layouts):
    """Row-major matrices are the transposed column-major view; a row-major C swaps the
    operands.  Checked against numpy on the logical matrices."""
    rng = np.random.default_rng(5)
    m, n, k = 130, 77, 95
    la, lb, lc = (sdk.ROW_MAJOR if ch == "R" else sdk.COLUMN_MAJOR for ch in layouts)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)     # logical op(A) = A (op N)
    B = rng.uniform(-1, 1, (n, k)).astype(np.float32)     # logical B, used with op T
    Cl = rng.uniform(-1, 1, (m, n)).astype(np.float32)

    def store(x, layout):  # bytes of x in the given layout, tight leading dimension
        return (np.ascontiguousarray(x) if layout == sdk.ROW_MAJOR
                else np.ascontiguousarray(x.T)), (x.shape[1] if layout == sdk.ROW_MAJOR
                                                  else x.shape[0])
    (sa, lda), (sb, ldb), (sc, ldc) = store(A, la), store(B, lb), store(Cl, lc)
    Ad, Bd, Cd = upload(s, sa), upload(s, sb), upload(s, sc)
    desc = s.gemm_desc(sdk.matrix(Ad, m, k, lda, la), sdk.matrix(Bd, n, k, ldb, lb),
                       sdk.matrix(Cd, m, n, ldc, lc), sdk.OP_N, sdk.OP_T, alpha=1.5, beta=0.5)
    plan = s.plan(desc)
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    got = download(Cd, sc.shape)
    got = got if lc == sdk.ROW_MAJOR else got.T
    ref = 1.5 * A.astype(np.float64) @ B.astype(np.float64).T + 0.5 * Cl
    assert float(np.max(np.abs(got - ref))) / k <= TOLERANCE


def test_tf32_compute_mode_uses_tensor_cores_within_tolerance(s):
    orc = load_oracle()
    m, n, k = 1024, 768, 2048
    a, b = orc.uniform(m * k, 31), orc.uniform(k * n, 32)
    A, B, Cm = upload(s, a), upload(s, b), s.alloc(4 * m * n)
    desc = s.gemm_desc(sdk.matrix(A, m, k, m), sdk.matrix(B, k, n, k), sdk.matrix(Cm, m, n, m),
                       mode=sdk.COMPUTE_FP32_TF32)
    plan = s.plan(desc)
    assert s.plan_info(plan).effective_compute_mode == sdk.COMPUTE_FP32_TF32
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    ref = orc.gemm(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
    assert normalized_error(download(Cm, (n, m)), ref, k, 1.0, 1.0) <= TOLERANCE


def test_plan_errors(s):
    A, C_ = s.alloc(4 * 64 * 64), s.alloc(4 * 64 * 64)
    ok = sdk.matrix(A, 64, 64, 64)
    out = C.c_void_p()
    for bad, status in [
        (s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=sdk.FP16), ok, sdk.matrix(C_, 64, 64, 64)),
         sdk.INVALID_ARGUMENT),                       # A and B types differ
        (s.gemm_desc(ok, ok, sdk.matrix(C_, 64, 64, 64), mode=sdk.COMPUTE_FP64),
         sdk.INVALID_ARGUMENT),                       # FP64 arithmetic on FP32 data
        (s.gemm_desc(ok, sdk.matrix(A, 32, 64, 64), sdk.matrix(C_, 64, 64, 64)),
         sdk.INVALID_ARGUMENT),                                   # k mismatch
        (s.gemm_desc(ok, ok, sdk.matrix(A, 64, 64, 64)), sdk.INVALID_ARGUMENT),  # C aliases A
        (s.gemm_desc(ok, ok, sdk.matrix(C_, 64, 64, 32)), sdk.INVALID_ARGUMENT),  # ld < rows
        (s.gemm_desc(ok, ok, sdk.matrix(C_, 64, 65, 64)), sdk.INVALID_ARGUMENT),  # out of bounds
    ]:
        assert s.t.gemm_plan_create(s.session, C.byref(bad), C.byref(out)) == status
        assert out.value is None
    d = s.gemm_desc(ok, ok, sdk.matrix(C_, 64, 64, 64))
    d.struct_size = 16
    assert s.t.gemm_plan_create(s.session, C.byref(d), C.byref(out)) == sdk.INCOMPATIBLE_ABI
    err = s.error()
    assert err.status == sdk.INCOMPATIBLE_ABI and err.stage == b"sdk"


def test_streamed_plan_under_a_small_budget():
    """A budget far below the operands makes the plan a panel schedule: several tiles,
    frames evicted and reused, and the same numbers as in place."""
    orc = load_oracle()
    m, n, k = 1536, 1280, 2048
    a, b, c = orc.uniform(m * k, 41), orc.uniform(k * n, 42), orc.uniform(m * n, 43)
    cfg = sdk.session_config(chunk_size_bytes=2 * MiB, cache_target_bytes=20 * MiB)
    with sdk.Sdk(cfg) as s:
        A, B, Cm = upload(s, a), upload(s, b), upload(s, c)
        desc = s.gemm_desc(sdk.matrix(A, k, m, k), sdk.matrix(B, n, k, n),
                           sdk.matrix(Cm, m, n, m), sdk.OP_T, sdk.OP_T, alpha=1.0, beta=1.0)
        plan = s.plan(desc)
        info = s.plan_info(plan)
        assert info.tile_count > 1 and info.maximum_working_set_bytes <= 20 * MiB
        op = C.c_void_p()
        s.check("gemm_submit", s.t.gemm_submit(plan, C.byref(op)))
        oi = s.wait(op.value)
        assert oi.state == sdk.COMPLETED and oi.result == sdk.SUCCESS
        assert oi.units_completed == oi.units_total == info.tile_count
        assert oi.bytes_h2d >= a.nbytes + b.nbytes
        s.t.operation_release(op.value)
        s.t.gemm_plan_release(plan)
        tel = s.telemetry()
        assert tel.handle_reuses > 0 and tel.mappings > tel.physical_handles_created
        ref = orc.gemm(1, 1, m, n, k, 1.0, a, k, b, n, 1.0, c, m)
        assert normalized_error(download(Cm, (n, m)), ref, k, 1.0, 1.0) <= TOLERANCE


def test_linear_bias_relu_through_a_transaction(s):
    """Linear + bias + ReLU: gemm_execute, then a transaction whose callback launches the
    library's bias/activation kernel on the resident output."""
    rng = np.random.default_rng(7)
    out_f, in_f, batch = 512, 384, 96
    W = (rng.standard_normal((out_f, in_f)) / np.sqrt(in_f)).astype(np.float32)  # row-major
    x = rng.uniform(-1, 1, (batch, in_f)).astype(np.float32)                    # row-major
    bias = rng.uniform(-0.5, 0.5, out_f).astype(np.float32)
    Wd, Xd, Bd = upload(s, W), upload(s, x), upload(s, bias)
    Yd = s.alloc(4 * out_f * batch)
    # Y (out_f x batch, column-major) = W (row-major out_f x in_f) * x^T
    desc = s.gemm_desc(sdk.matrix(Wd, out_f, in_f, in_f, sdk.ROW_MAJOR),
                       sdk.matrix(Xd, batch, in_f, in_f, sdk.ROW_MAJOR),
                       sdk.matrix(Yd, out_f, batch, out_f), sdk.OP_N, sdk.OP_T)
    plan = s.plan(desc)
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    seen = {}

    def body(ctx):
        y, b = ctx.ranges[0], ctx.ranges[1]
        seen["ranges"] = ctx.range_count
        seen["stream"] = ctx.native_stream
        return sdk.bias_activation(y.device_address, out_f, out_f, batch, b.device_address, True,
                                   ctx.native_stream)
    d = s.transaction_desc([(Yd, 0, Yd.size, sdk.READ_WRITE), (Bd, 0, Bd.size, sdk.READ)], body)
    s.check("transaction_execute", s.t.transaction_execute(s.session, C.byref(d),
                                                           sdk.TIMEOUT_INFINITE))
    assert seen["ranges"] == 2 and seen["stream"] != 0
    got = download(Yd, (batch, out_f))
    ref = np.maximum(x.astype(np.float64) @ W.astype(np.float64).T + bias, 0.0)
    assert float(np.max(np.abs(got - ref))) <= 1e-5 * in_f ** 0.5
    assert s.telemetry().transactions_completed >= 1


def test_transaction_callback_failure_is_reported(s):
    Y = s.alloc(4096)

    def body(ctx):
        return sdk.CALLBACK_FAILED
    d = s.transaction_desc([(Y, 0, 4096, sdk.READ)], body)
    assert s.t.transaction_execute(s.session, C.byref(d), sdk.TIMEOUT_INFINITE) == \
        sdk.CALLBACK_FAILED
    err = s.error()
    assert err.status == sdk.CALLBACK_FAILED and err.native_domain == 4  # CALLBACK
    # the session stays usable
    Y.write(np.ones(1024, dtype=np.float32))
    assert np.all(download(Y, 1024) == 1.0)
    # workspace above the session cap is rejected at submission
    d = s.transaction_desc([(Y, 0, 4096, sdk.READ)], lambda ctx: 0, workspace_bytes=8 * MiB)
    out = C.c_void_p()
    assert s.t.transaction_submit(s.session, C.byref(d), C.byref(out)) == sdk.INVALID_ARGUMENT


def test_prefetch_makes_the_gemm_a_cache_hit():
    orc = load_oracle()
    m = n = k = 1024
    cfg = sdk.session_config(chunk_size_bytes=2 * MiB, cache_target_bytes=64 * MiB)
    with sdk.Sdk(cfg) as s:
        a, b = orc.uniform(m * k, 51), orc.uniform(k * n, 52)
        A, B, Cm = upload(s, a), upload(s, b), s.alloc(4 * m * n)
        filler = [s.alloc(16 * MiB) for _ in range(4)]  # pushes A and B out of the cache
        for f in filler:
            f.write(np.zeros(4 * MiB, dtype=np.float32))
        desc = s.gemm_desc(sdk.matrix(A, m, k, m), sdk.matrix(B, k, n, k), sdk.matrix(Cm, m, n, m))
        plan = s.plan(desc)
        pd = s.prefetch_desc([(A, 0, A.size, sdk.READ), (B, 0, B.size, sdk.READ)])
        op = C.c_void_p()
        s.check("prefetch_submit", s.t.prefetch_submit(s.session, C.byref(pd), C.byref(op)))
        assert s.wait(op.value).state == sdk.COMPLETED
        s.t.operation_release(op.value)
        s.check("gemm_submit", s.t.gemm_submit(plan, C.byref(op)))
        oi = s.wait(op.value)
        assert oi.state == sdk.COMPLETED
        assert oi.bytes_h2d == 0  # A and B were already resident (or on their way)
        s.t.operation_release(op.value)
        s.t.gemm_plan_release(plan)
        ref = orc.gemm(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
        assert normalized_error(download(Cm, (n, m)), ref, k, 1.0, 1.0) <= TOLERANCE


def test_operation_lifecycle_cancel_deadline_busy(s):
    """A callback that holds the worker makes the queue observable: the next operation
    can be cancelled, a deadline passes in the queue, the running one answers BUSY."""
    Y = s.alloc(4096)
    gate = threading.Event()

    def hold(ctx):
        gate.wait(10.0)
        return 0
    d1 = s.transaction_desc([(Y, 0, 4096, sdk.READ)], hold)
    op1, op2, op3 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    s.check("submit", s.t.transaction_submit(s.session, C.byref(d1), C.byref(op1)))
    d2 = s.transaction_desc([(Y, 0, 4096, sdk.READ)], lambda ctx: 0)
    s.check("submit", s.t.transaction_submit(s.session, C.byref(d2), C.byref(op2)))
    d3 = s.transaction_desc([(Y, 0, 4096, sdk.READ)], lambda ctx: 0, deadline_ms=20)
    s.check("submit", s.t.transaction_submit(s.session, C.byref(d3), C.byref(op3)))
    info = sdk.OperationInfo(struct_size=C.sizeof(sdk.OperationInfo))
    for _ in range(500):  # until the worker is inside op1's callback
        s.t.operation_poll(op1.value, C.byref(info))
        if info.state == sdk.RUNNING:
            break
        time.sleep(0.01)
    assert info.state == sdk.RUNNING
    assert s.t.operation_cancel(op1.value) == sdk.BUSY
    assert s.t.operation_wait(op1.value, 10, C.byref(info)) == sdk.TIMEOUT
    assert s.t.operation_cancel(op2.value) == sdk.SUCCESS
    assert s.t.session_drain(s.session, 10) == sdk.TIMEOUT
    time.sleep(0.05)  # op3's deadline passes while it waits in the queue
    gate.set()
    assert s.wait(op1.value).state == sdk.COMPLETED
    i2 = s.wait(op2.value)
    assert (i2.state, i2.result) == (sdk.OP_CANCELLED, sdk.CANCELLED)
    i3 = s.wait(op3.value)
    assert (i3.state, i3.result) == (sdk.FAILED, sdk.TIMEOUT)
    assert s.op_error(op3.value).status == sdk.TIMEOUT
    assert s.t.session_drain(s.session, sdk.TIMEOUT_INFINITE) == sdk.SUCCESS
    for op in (op1, op2, op3):
        s.t.operation_release(op.value)


def test_released_allocation_fails_a_plan_and_handles_outlive_close():
    cfg = sdk.session_config()
    s = sdk.Sdk(cfg)
    A, Cm = s.alloc(4 * 32 * 32), s.alloc(4 * 32 * 32)
    plan = s.plan(s.gemm_desc(sdk.matrix(A, 32, 32, 32), sdk.matrix(A, 32, 32, 32),
                              sdk.matrix(Cm, 32, 32, 32)))
    keep = s.alloc(1024)
    assert A.release() == sdk.SUCCESS
    assert s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE) == sdk.INVALID_ARGUMENT
    s.t.gemm_plan_release(plan)
    t = s.t
    assert t.session_close(s.session, sdk.TIMEOUT_INFINITE) == sdk.SUCCESS
    assert t.session_close(s.session, sdk.TIMEOUT_INFINITE) == sdk.SUCCESS  # idempotent
    out = C.c_void_p()
    d = sdk.AllocationDesc(struct_size=C.sizeof(sdk.AllocationDesc), size_bytes=64)
    assert t.allocation_create(s.session, C.byref(d), C.byref(out)) == sdk.CLOSED
    assert keep.release() == sdk.SUCCESS and Cm.release() == sdk.SUCCESS
    t.session_release(s.session)
    s.session = C.c_void_p()


def test_sdk_calls_from_a_callback_answer_busy(s):
    """A transaction callback runs on the session's worker: synchronous SDK calls from it
    could never run (they queue behind the callback), so they answer BUSY."""
    Y = s.alloc(4096)
    seen = {}

    def body(ctx):
        buf = np.zeros(4, dtype=np.float32)
        seen["read"] = s.t.allocation_read(Y.handle, 0, buf.ctypes.data, 16)
        seen["drain"] = s.t.session_drain(s.session, 0)
        seen["close"] = s.t.session_close(s.session, 0)
        return 0
    d = s.transaction_desc([(Y, 0, 4096, sdk.READ)], body)
    s.check("transaction_execute", s.t.transaction_execute(s.session, C.byref(d),
                                                           sdk.TIMEOUT_INFINITE))
    assert seen == {"read": sdk.BUSY, "drain": sdk.BUSY, "close": sdk.BUSY}
    Y.write(np.ones(1024, dtype=np.float32))  # still open and working
    assert np.all(download(Y, 1024) == 1.0)


def test_process_exits_cleanly_with_a_session_left_open():
    """A session that its owner never closes keeps a budget-sampler thread that queries
    the device every budget_poll_ms.  At process exit the library stops such samplers
    before the CUDA runtime tears its state down, so the process ends with status 0 (a
    sampler still querying a torn-down runtime could crash the exit)."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, numpy as np\n"
        f"sys.path.insert(0, {str(root)!r})\n"
        "from xvram_b200 import sdk\n"
        "s = sdk.Sdk(sdk.session_config(budget_poll_ms=1))\n"
        "a = s.alloc(1 << 20)\n"
        "a.write(np.ones(1 << 18, dtype=np.float32))\n"
        "print('left open')\n")
    for _ in range(3):
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                           timeout=120)
        assert r.returncode == 0 and "left open" in r.stdout, (r.returncode, r.stderr[-2000:])
