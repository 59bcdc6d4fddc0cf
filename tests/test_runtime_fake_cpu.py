"""The residency runtime, out-of-core executor, SDK and compat adapter on the host-memory
fake device (tests/fake_device): the real library code paths -- frame pool, chunk states,
eviction, write-back, the streamed panel replay, transactions, prefetch, the live budget,
failure poisoning -- checked on the CPU, the way the reference's fake-driver unit tests
drive its runtime (reference tests/unit/residency_executor_fake_tests.cpp,
vmm_executor_fake_tests.cpp).  The fake's GEMM is a plain FP32 loop in test code."""
from __future__ import annotations

import ctypes as C
import subprocess
import sys

import numpy as np
import pytest

from fake_device import installed
from oracle_lib import TOLERANCE, load_oracle, normalized_error

from xvram_b200 import sdk

MiB = 1 << 20


def session(budget=0, chunk=2 * MiB, poll=100, headroom=512 * MiB):
    return sdk.Sdk(sdk.session_config(cache_target_bytes=budget, chunk_size_bytes=chunk,
                                      budget_poll_ms=poll, device_headroom_bytes=headroom))


def upload(s, arr):
    a = s.alloc(arr.nbytes)
    a.write(np.ascontiguousarray(arr))
    return a


def download(alloc, count):
    out = np.empty(count, dtype=np.float32)
    alloc.read(out)
    return out


def run_gemm(s, op_a, op_b, m, n, k, alpha, beta, seed):
    orc = load_oracle()
    a, b, c = orc.uniform(m * k, seed), orc.uniform(k * n, seed + 1), orc.uniform(m * n, seed + 2)
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    A, B, Cm = upload(s, a), upload(s, b), upload(s, c)
    desc = s.gemm_desc(sdk.matrix(A, m if op_a == 0 else k, k if op_a == 0 else m, lda),
                       sdk.matrix(B, k if op_b == 0 else n, n if op_b == 0 else k, ldb),
                       sdk.matrix(Cm, m, n, m), op_a, op_b, alpha=alpha, beta=beta,
                       mode=sdk.COMPUTE_FP32_STRICT)
    plan = s.plan(desc)
    info = s.plan_info(plan)
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    out = download(Cm, m * n).reshape(n, m)
    ref = orc.gemm(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, m)
    return normalized_error(out, ref, k, 1.0, 1.0), info


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_in_place_gemm(op_a, op_b):
    with installed(), session() as s:
        err, info = run_gemm(s, op_a, op_b, 150, 90, 70, 0.5, 1.5, 3)
        assert info.tile_count == 1 and err <= TOLERANCE


@pytest.mark.parametrize("op_a,op_b", [(0, 1), (1, 0)])
def test_streamed_gemm_under_a_small_budget(op_a, op_b):
    """18.5 MiB of operands (plus the transposes' workspace for TN) through a 16 MiB budget
    of 2 MiB frames: a panel schedule (of blocks smaller than one wave -- the only ones
    that fit) with evictions and frame reuse, the same result as in place."""
    with installed(), session(budget=16 * MiB) as s:
        err, info = run_gemm(s, op_a, op_b, 1536, 1280, 1024, 1.0, 1.0, 9)
        assert info.tile_count > 1 and info.maximum_working_set_bytes <= 16 * MiB
        assert err <= TOLERANCE
        tel = s.telemetry()
        assert tel.handle_reuses > 0 and tel.mappings > tel.physical_handles_created
        assert tel.resident_bytes_peak <= 16 * MiB


def test_dirty_chunks_survive_eviction():
    """Eight 2 MiB allocations and a 6 MiB pool: the first three are written straight to
    device frames (dirty), the rest to host backing once the pool is full (writes never
    evict).  Prefetching the host-backed ones then evicts the dirty frames, which are
    written back first; every read returns its own pattern."""
    with installed(), session(budget=6 * MiB) as s:
        blocks = []
        for i in range(8):
            a = s.alloc(2 * MiB)
            a.write(np.full(512 * 1024, float(i + 1), dtype=np.float32))
            blocks.append(a)
        d = s.prefetch_desc([(a, 0, 2 * MiB, sdk.READ) for a in blocks[5:]])
        op = C.c_void_p()
        s.check("prefetch", s.t.prefetch_submit(s.session, C.byref(d), C.byref(op)))
        assert s.wait(op.value).result == sdk.SUCCESS
        s.t.operation_release(op.value)
        for i, a in enumerate(blocks):
            assert np.all(download(a, 512 * 1024) == i + 1)
        tel = s.telemetry()
        assert tel.dirty_evictions > 0 and tel.writebacks_completed == tel.dirty_evictions
        assert tel.resident_bytes_peak <= 6 * MiB


def test_transaction_writes_reach_the_host_after_eviction():
    """A read-write transaction marks its chunks dirty: after they are evicted by other
    traffic, the host copy holds what the callback wrote."""
    with installed(), session(budget=6 * MiB) as s:
        y = s.alloc(2 * MiB)
        y.write(np.zeros(512 * 1024, dtype=np.float32))

        def body(ctx):  # the fake's device addresses are host addresses
            n = ctx.ranges[0].length_bytes // 4
            arr = (C.c_float * n).from_address(ctx.ranges[0].device_address)
            for i in range(0, n, 4096):
                arr[i] = 42.0
            return 0
        d = s.transaction_desc([(y, 0, 2 * MiB, sdk.READ_WRITE)], body)
        s.check("transaction", s.t.transaction_execute(s.session, C.byref(d), sdk.TIMEOUT_INFINITE))
        others = [s.alloc(2 * MiB) for _ in range(4)]
        for o in others:
            o.write(np.ones(512 * 1024, dtype=np.float32))
        out = download(y, 512 * 1024)
        assert np.all(out[::4096] == 42.0) and out[1] == 0.0
        assert s.telemetry().transactions_completed >= 1


def test_write_only_transaction_skips_the_upload():
    with installed(), session(budget=64 * MiB) as s:
        y = s.alloc(4 * MiB)
        y.write(np.ones(MiB, dtype=np.float32))
        filler = [s.alloc(16 * MiB) for _ in range(4)]
        for f in filler:  # push y out of the pool
            f.write(np.zeros(4 * MiB, dtype=np.float32))
        before = s.telemetry().bytes_h2d
        d = s.transaction_desc([(y, 0, 4 * MiB, sdk.WRITE_ONLY)], lambda ctx: 0)
        s.check("transaction", s.t.transaction_execute(s.session, C.byref(d), sdk.TIMEOUT_INFINITE))
        assert s.telemetry().bytes_h2d == before  # nothing uploaded for a whole-chunk write


def test_live_budget_on_the_fake():
    with installed(free_bytes=64 * MiB) as fake, session(poll=1, headroom=0) as s:
        blocks = [s.alloc(2 * MiB) for _ in range(12)]
        for i, a in enumerate(blocks):
            a.write(np.full(512 * 1024, float(i), dtype=np.float32))
        t0 = s.telemetry()
        fake.fake_device_set_memory(0, 16 << 30)  # someone took everything else

        def touch():
            import time
            time.sleep(0.002)
            d = s.prefetch_desc([(blocks[-1], 0, 4096, sdk.READ)])
            op = C.c_void_p()
            s.check("prefetch", s.t.prefetch_submit(s.session, C.byref(d), C.byref(op)))
            s.wait(op.value)
            s.t.operation_release(op.value)
        touch()
        t1 = s.telemetry()
        assert t1.budget_shrinks == t0.budget_shrinks + 1
        assert t1.cache_target_bytes <= 24 * MiB  # free 0 + the frames it holds
        for i, a in enumerate(blocks):
            assert np.all(download(a, 512 * 1024)[::8192] == i)
        fake.fake_device_set_memory(64 * MiB, 16 << 30)
        for _ in range(4):
            touch()
        assert s.telemetry().budget_grows >= 1


def test_budget_samples_come_from_the_sampler_thread():
    """With a 50 ms poll, free memory is sampled by a thread of the runtime's own, with no
    operation running (budget_sample_count grows while the session is idle); an operation
    applies the newest sample it has not applied yet, so a change is acted on by the first
    operation after the sampler has seen it."""
    import time
    with installed(free_bytes=64 * MiB) as fake, session(poll=50, headroom=0) as s:
        blocks = [s.alloc(2 * MiB) for _ in range(12)]
        for i, a in enumerate(blocks):
            a.write(np.full(512 * 1024, float(i), dtype=np.float32))

        def touch():
            d = s.prefetch_desc([(blocks[-1], 0, 4096, sdk.READ)])
            op = C.c_void_p()
            s.check("prefetch", s.t.prefetch_submit(s.session, C.byref(d), C.byref(op)))
            s.wait(op.value)
            s.t.operation_release(op.value)

        touch()
        n0 = s.telemetry().budget_sample_count
        time.sleep(0.4)                     # idle: the sampler keeps sampling
        touch()                             # the operation takes in every sample since
        t1 = s.telemetry()
        assert t1.budget_sample_count >= n0 + 3
        assert t1.budget_shrinks == 0
        fake.fake_device_set_memory(0, 16 << 30)
        time.sleep(0.2)                     # several polls: the sampler has seen it
        touch()
        t2 = s.telemetry()
        assert t2.budget_shrinks == 1
        assert t2.cache_target_bytes <= 24 * MiB
        for i, a in enumerate(blocks):
            assert np.all(download(a, 512 * 1024)[::8192] == i)


def test_injected_copy_failure_poisons_the_session():
    with installed() as fake, session() as s:
        a = s.alloc(4 * MiB)
        b = s.alloc(4 * MiB)
        a.write(np.ones(MiB, dtype=np.float32))
        fake.fake_device_fail(b"sgemm", 0)
        desc = s.gemm_desc(sdk.matrix(a, 1024, 1024, 1024), sdk.matrix(a, 1024, 1024, 1024),
                           sdk.matrix(b, 1024, 1024, 1024))
        plan = s.plan(desc)
        assert s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE) == sdk.CUDA_ERROR
        err = s.error()
        assert err.status == sdk.CUDA_ERROR and err.native_name == b"injected"
        assert s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE) == sdk.POISONED
        assert s.telemetry().poisoned == 1
        s.t.gemm_plan_release(plan)


COMPAT_SCRIPT = r"""
import sys
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
from fake_device import installed
from oracle_lib import load_oracle, normalized_error
from xvram_b200 import compat as cp
with installed():
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.chunk_size_bytes = 2 << 20
    cfg.session.cache_target_bytes = 16 << 20
    api.check("initialize", api.initialize(cfg))
    orc = load_oracle()
    m, n, k = 1536, 1280, 1024
    a, b, c = orc.uniform(m * k, 1), orc.uniform(k * n, 2), orc.uniform(m * n, 3)
    ptrs = [api.malloc(x.nbytes) for x in (a, b, c)]
    for p, x in zip(ptrs, (a, b, c)):
        api.h2d(p, x.ctypes.data, x.nbytes)
    h = api.blas_create()
    api.check("sgemm", api.sgemm(h, 1, 0, m, n, k, 0.5, ptrs[0], k, ptrs[1], k, 1.5, ptrs[2], m))
    out = np.empty(m * n, np.float32)
    api.d2h(out.ctypes.data, ptrs[2], out.nbytes)
    ref = orc.gemm(1, 0, m, n, k, 0.5, a, k, b, k, 1.5, c, m)
    err = normalized_error(out.reshape(n, m), ref, k, 1.0, 1.0)
    tel = api.telemetry()
    api.shutdown()
    print(err, tel.runtime.handle_reuses, tel.tiles_retired)
"""


def test_compat_adapter_on_the_fake():
    """The compat table (one initialisation per process, so in a child): memcpy, an
    out-of-core blas_sgemm (18.5 MiB of operands and the transposes' workspace) through
    a 16 MiB budget, memcpy back."""
    from fake_device import ROOT
    r = subprocess.run([sys.executable, "-c", COMPAT_SCRIPT, str(ROOT)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    err, reuses, tiles = r.stdout.split()
    assert float(err) <= TOLERANCE and int(reuses) > 0 and int(tiles) > 1


@pytest.mark.parametrize("policy", ["clock", "lru"])
def test_victim_policy_clock_spares_dirty_lru_takes_oldest(policy):
    """Four 2 MiB frames hold A0..A3, each written while resident (dirty on the device).
    A4 and A5 are written while the pool is full, so they stay host-side.  Prefetching A4
    evicts one of A0..A3 and uploads A4, which is then resident and clean.  Prefetching A5
    needs a frame again: LRU evicts the least recently used chunk, one of A0..A3, writing
    it back first (a dirty eviction); CLOCK, the reference's default (reference
    src/residency/policy.cpp:17-28), takes its victim from the cheapest cost class --
    clean before dirty -- so it evicts A4 without a write-back."""
    code = {"clock": sdk.CACHE_POLICY_CLOCK, "lru": sdk.CACHE_POLICY_LRU}[policy]
    cfg = sdk.session_config(cache_target_bytes=8 * MiB, chunk_size_bytes=2 * MiB,
                             device_headroom_bytes=512 * MiB, cache_policy=code)
    with installed(), sdk.Sdk(cfg) as s:
        blocks = []
        for i in range(6):
            a = s.alloc(2 * MiB)
            a.write(np.full(MiB // 2, float(i + 1), dtype=np.float32))
            blocks.append(a)

        def prefetch(a):
            d = s.prefetch_desc([(a, 0, 2 * MiB, sdk.READ)])
            op = C.c_void_p()
            s.check("prefetch", s.t.prefetch_submit(s.session, C.byref(d), C.byref(op)))
            assert s.wait(op.value).result == sdk.SUCCESS
            s.t.operation_release(op.value)

        prefetch(blocks[4])
        t0 = s.telemetry()
        prefetch(blocks[5])
        t1 = s.telemetry()
        delta = (t1.clean_evictions - t0.clean_evictions, t1.dirty_evictions - t0.dirty_evictions)
        assert delta == ((1, 0) if policy == "clock" else (0, 1)), delta
        assert t1.handle_reuses == t0.handle_reuses + 1
        for i, a in enumerate(blocks):                       # nothing lost either way
            assert download(a, MiB // 2)[0] == i + 1
        t2 = s.telemetry()
        assert t2.event_boundaries == t2.unmaps
