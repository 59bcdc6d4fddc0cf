"""End-to-end scenarios through the compat C table, one per process.

The table admits one initialisation per process (reference
include/xvram/cuda_compat.h:30-32), so tests/test_compat_gpu.py runs each scenario as
`python tests/compat_scenarios.py <name>` and reads the JSON it prints last.
"""
from __future__ import annotations

import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))

from oracle_lib import TOLERANCE, load_oracle, normalized_error, reference_criterion  # noqa: E402
from xvram_b200 import compat as cp  # noqa: E402

MiB = 1 << 20


def ptr(x: np.ndarray) -> int:
    return x.ctypes.data


def init(api: cp.CompatApi, cache_target: int = 0, chunk: int = 64 * MiB) -> None:
    cfg = cp.compat_config_init()
    cfg.session.cache_target_bytes = cache_target
    cfg.session.chunk_size_bytes = chunk
    api.check("initialize", api.initialize(cfg))


def upload(api, arr: np.ndarray) -> int:
    d = api.malloc(arr.nbytes)
    api.h2d(d, ptr(arr), arr.nbytes)
    return d


def scenario_preview(oracle):
    """examples/preview-gemm/main.cpp flow: 37x19x67 NN through the table."""
    api = cp.CompatApi()
    m, n, k = 37, 19, 67
    a = np.array([[oracle.lib.xo_pv_a(r, c) for r in range(m)] for c in range(k)], np.float32)
    b = np.array([[oracle.lib.xo_pv_b(r, c) for r in range(k)] for c in range(n)], np.float32)
    c = np.zeros((n, m), np.float32)
    init(api)
    da, db, dc = upload(api, a), upload(api, b), upload(api, c)
    h = api.blas_create()
    api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 1.0, da, m, db, k, 0.0, dc, m))
    out = np.empty_like(c)
    api.d2h(ptr(out), dc, out.nbytes)
    ref = oracle.gemm(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
    api.blas_destroy(h)
    for d in (dc, db, da):
        api.free(d)
    t = api.telemetry()
    res = dict(ok=reference_criterion(out, ref), max_abs=float(np.abs(out - ref).max()),
               gemm_calls=t.gemm_calls, live_allocations=t.live_allocations,
               live_handles=t.live_handles)
    res["shutdown"] = api.shutdown()
    t = api.telemetry()
    res.update(state=t.state, cleanup_completed=t.cleanup_completed)
    return res


def scenario_padded(oracle):
    """The reference's padded gate suite: 37x19x67, padding 5, offset 11, NN/NT/TN/TT,
    interior pointers, padding value -1234.5 preserved bit for bit."""
    import json as _json
    golden = _json.loads((HERE / "golden" / "reference_vectors.json").read_text())
    g = golden["cb_padded_fills"]
    shp = g["shape"]
    m, n, k, off = shp["m"], shp["n"], shp["k"], shp["offset"]
    fills = {(f["ta"], f["tb"], f["operand"]): f for f in g["fills"]}
    api = cp.CompatApi()
    init(api)
    h = api.blas_create()
    results = {}
    for ta in (0, 1):
        for tb in (0, 1):
            arrs, lds, devs = [], [], []
            for operand in range(3):
                f = fills[(ta, tb, operand)]
                arr = np.frombuffer(bytes.fromhex(f["bits"]), dtype=np.float32).copy()
                arrs.append(arr)
                lds.append(f["ld"])
                devs.append(upload(api, arr))
            for alpha, beta in ((1.0, 0.0), (0.5, 1.5)):
                st = api.sgemm(h, ta, tb, m, n, k, alpha, devs[0] + 4 * off, lds[0],
                               devs[1] + 4 * off, lds[1], beta, devs[2] + 4 * off, lds[2])
                api.check("sgemm", st)
                out = np.empty_like(arrs[2])
                api.d2h(ptr(out), devs[2], out.nbytes)
                ref = oracle.gemm(ta, tb, m, n, k, alpha, arrs[0][off:], lds[0], arrs[1][off:],
                                  lds[1], beta, arrs[2][off:], lds[2])
                ldc = lds[2]
                body = np.stack([out[off + j * ldc: off + j * ldc + m] for j in range(n)])
                mask = np.ones_like(out, bool)
                for j in range(n):
                    mask[off + j * ldc: off + j * ldc + m] = False
                ok = reference_criterion(body, ref) and np.array_equal(out[mask], arrs[2][mask])
                results[f"{ta}{tb}_{alpha}_{beta}"] = bool(ok)
                # next pass starts from the current C
                api.h2d(devs[2], ptr(arrs[2]), arrs[2].nbytes)
            for d in devs:
                api.free(d)
    api.blas_destroy(h)
    results["shutdown"] = api.shutdown()
    return results


def scenario_errors(oracle):
    """Lifecycle and preflight error classes of the adapter."""
    api = cp.CompatApi()
    r = {}
    out = C.c_void_p()
    r["before_init"] = api.t.malloc_device(C.byref(out), 16)
    bad = cp.compat_config_init()
    bad.flags = 1
    r["bad_config"] = api.initialize(bad)
    bad = cp.compat_config_init()
    bad.session.chunk_size_bytes = 3 << 20
    r["bad_chunk"] = api.initialize(bad)
    init(api)
    a = np.ones((64, 64), np.float32)
    da, db, dc = upload(api, a), upload(api, a), upload(api, a)
    h = api.blas_create()
    r["ok"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, da, 64, db, 64, 0.0, dc, 64)
    r["ld_small"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, da, 63, db, 64, 0.0, dc, 64)
    r["bad_op"] = api.sgemm(h, 2, 0, 64, 64, 64, 1.0, da, 64, db, 64, 0.0, dc, 64)
    r["zero_m"] = api.sgemm(h, 0, 0, 0, 64, 64, 1.0, da, 64, db, 64, 0.0, dc, 64)
    r["alias"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, da, 64, db, 64, 0.0, da, 64)
    r["foreign"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, ptr(a), 64, db, 64, 0.0, dc, 64)
    r["misaligned"] = api.sgemm(h, 0, 0, 8, 8, 8, 1.0, da + 2, 64, db, 64, 0.0, dc, 64)
    r["oob"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, da + 4, 64, db, 64, 0.0, dc, 64)
    r["nan_alpha"] = api.sgemm(h, 0, 0, 64, 64, 64, float("nan"), da, 64, db, 64, 0.0, dc, 64)
    r["bad_handle"] = api.sgemm(ptr(a), 0, 0, 64, 64, 64, 1.0, da, 64, db, 64, 0.0, dc, 64)
    r["set_device_other"] = api.t.set_device(1)
    r["set_stream"] = api.t.blas_set_stream(h, 1234)
    r["pointer_mode_device"] = api.t.blas_set_pointer_mode(h, 1)
    r["math_tensor_op"] = api.t.blas_set_math_mode(h, 1)
    r["math_tf32"] = api.t.blas_set_math_mode(h, 3)
    r["math_pedantic"] = api.t.blas_set_math_mode(h, 2)
    r["free_interior"] = api.t.free_device(da + 64)
    r["memcpy_d2d"] = api.t.memcpy(da, db, 64, 3)
    r["memcpy_oob"] = api.t.memcpy(da, ptr(a), a.nbytes + 4, cp.H2D)
    r["memcpy_host_is_managed"] = api.t.memcpy(da, db, 64, cp.H2D)
    r["free_null"] = api.t.free_device(None)
    r["free"] = api.t.free_device(da)
    r["double_free"] = api.t.free_device(da)
    r["use_after_free"] = api.sgemm(h, 0, 0, 64, 64, 64, 1.0, da, 64, db, 64, 0.0, dc, 64)
    r["shutdown"] = api.shutdown()
    r["after_shutdown"] = api.t.malloc_device(C.byref(out), 16)
    r["second_init"] = api.initialize()
    t = api.telemetry()
    r["state"] = t.state
    r["attempted_eq"] = t.calls_attempted == t.calls_completed + t.calls_rejected
    return r


def scenario_out_of_core(oracle):
    """Operands larger than the device budget: the streamed path with real eviction and
    frame reuse, two passes like the reference's oversubscription gates."""
    api = cp.CompatApi()
    m = n = k = 6144
    init(api, cache_target=512 * MiB, chunk=64 * MiB)
    a = oracle.uniform(m * k, 30).reshape(k, m)       # op N: m x k
    b = oracle.uniform(n * k, 31).reshape(k, n)       # op T: stored n x k
    c = oracle.uniform(m * n, 32).reshape(n, m)
    da, db, dc = upload(api, a), upload(api, b), upload(api, c)
    h = api.blas_create()
    alpha, beta = 1.0, 1.0
    for _ in range(2):
        api.check("sgemm", api.sgemm(h, 0, 1, m, n, k, alpha, da, m, db, n, beta, dc, m))
    out = np.empty_like(c)
    api.d2h(ptr(out), dc, out.nbytes)
    rng = np.random.default_rng(1)
    rows, cols = rng.integers(0, m, 20000), rng.integers(0, n, 20000)
    dot = oracle.gemm_sampled(0, 1, k, 1.0, a, m, b, n, 0.0, None, m, rows, cols, threads=16)
    cin = c[cols, rows].astype(np.float64)
    ref = alpha * dot + beta * (alpha * dot + beta * cin)
    err = float(np.max(np.abs(out[cols, rows] - ref))) / (2 * k)
    t = api.telemetry()
    info = cp.runtime_info()
    res = dict(err=err, ok=err <= TOLERANCE,
               streamed=info.gemm_streamed, in_place=info.gemm_in_place,
               block=(info.last_block_m, info.last_block_n, info.last_panel_k),
               steps=info.last_steps, slots=info.last_panel_slots,
               tiles_submitted=t.tiles_submitted, tiles_retired=t.tiles_retired,
               clean_evictions=t.runtime.clean_evictions, dirty_evictions=t.runtime.dirty_evictions,
               handle_reuses=t.runtime.handle_reuses, mappings=t.runtime.mappings,
               unmaps=t.runtime.unmaps, bytes_h2d=t.runtime.bytes_h2d,
               bytes_d2h=t.runtime.bytes_d2h, cache_target=t.runtime.cache_target_bytes,
               resident_peak=t.runtime.resident_bytes_peak,
               panel_slot_refills=info.panel_slot_refills)
    res["shutdown"] = api.shutdown()
    t = api.telemetry()
    res["mappings_end"], res["unmaps_end"] = t.runtime.mappings, t.runtime.unmaps
    res["event_boundaries_end"] = t.runtime.event_boundaries
    return res


def scenario_in_place_two_passes(oracle):
    api = cp.CompatApi()
    m, n, k = 2048, 1536, 1024
    init(api)
    a = oracle.uniform(m * k, 40).reshape(m, k)   # op T: stored k x m
    b = oracle.uniform(k * n, 41).reshape(n, k)   # op N: stored k x n
    c = oracle.uniform(m * n, 42).reshape(n, m)
    da, db, dc = upload(api, a), upload(api, b), upload(api, c)
    h = api.blas_create()
    for _ in range(2):
        api.check("sgemm", api.sgemm(h, 1, 0, m, n, k, 0.5, da, k, db, k, 1.5, dc, m))
    out = np.empty_like(c)
    api.d2h(ptr(out), dc, out.nbytes)
    dot = oracle.gemm(1, 0, m, n, k, 1.0, a, k, b, k, 0.0, None, m, threads=16)
    ref = 0.5 * dot + 1.5 * (0.5 * dot + 1.5 * c.astype(np.float64))
    err = float(np.max(np.abs(out - ref))) / (2 * k)
    info = cp.runtime_info()
    res = dict(err=err, ok=err <= TOLERANCE, in_place=info.gemm_in_place,
               streamed=info.gemm_streamed)
    res["shutdown"] = api.shutdown()
    return res


def scenario_tensor_cores(oracle):
    """Math mode 3 (TF32 tensor-op math) selects the three-term TF32 tcgen05 path, in place
    and out of core (512 MiB budget), both within the stated tolerance."""
    api = cp.CompatApi()
    init(api, cache_target=512 * MiB, chunk=64 * MiB)
    h = api.blas_create()
    api.check("math", api.t.blas_set_math_mode(h, 3))
    mode = C.c_uint32(0)
    api.check("get_math", api.t.blas_get_math_mode(h, C.byref(mode)))
    res = {"mode": mode.value}
    for tag, (m, n, k) in (("in_place", (1024, 768, 1536)), ("streamed", (6144, 6144, 6144))):
        a = oracle.uniform(m * k, 60).reshape(m, k)   # op T: stored k x m
        b = oracle.uniform(k * n, 61).reshape(n, k)   # op N: stored k x n
        c = oracle.uniform(m * n, 62).reshape(n, m)
        da, db, dc = upload(api, a), upload(api, b), upload(api, c)
        api.check("sgemm", api.sgemm(h, 1, 0, m, n, k, 0.5, da, k, db, k, 1.5, dc, m))
        out = np.empty_like(c)
        api.d2h(ptr(out), dc, out.nbytes)
        rng = np.random.default_rng(2)
        rows, cols = rng.integers(0, m, 8192), rng.integers(0, n, 8192)
        ref = oracle.gemm_sampled(1, 0, k, 0.5, a, k, b, k, 1.5, c, m, rows, cols, threads=16)
        res[tag] = float(np.max(np.abs(out[cols, rows] - ref))) / k
        for d in (da, db, dc):
            api.free(d)
    info = cp.runtime_info()
    res.update(in_place_calls=info.gemm_in_place, streamed_calls=info.gemm_streamed,
               ok=max(res["in_place"], res["streamed"]) <= TOLERANCE)
    res["shutdown"] = api.shutdown()
    return res


def scenario_deferred(oracle):
    """blas_sgemm returning before its kernels finish (the default): C split into column
    blocks, each copied home after its own kernel.  Every operation with ldc > m, C read
    whole and in pieces that cut through blocks; digests of C for comparison with a run
    under XVRAM_B200_SYNC_GEMM=1, and sampled FP64 errors."""
    import hashlib
    api = cp.CompatApi()
    init(api)
    h = api.blas_create()
    m, n, k = 8192, 4096, 256
    ldc = m + 8
    res = {"digests": {}, "errors": {}}
    rng = np.random.default_rng(5)
    rows, cols = rng.integers(0, m, 8192), rng.integers(0, n, 8192)
    for op_a, op_b, math in [(x, y, z) for z in (0, 3) for x in (0, 1) for y in (0, 1)]:
        api.check("math", api.t.blas_set_math_mode(h, math))
        lda = m if op_a == 0 else k
        ldb = k if op_b == 0 else n
        a = oracle.uniform(lda * (k if op_a == 0 else m), 70 + op_a)
        b = oracle.uniform(ldb * (n if op_b == 0 else k), 72 + op_b)
        c = oracle.uniform(ldc * n, 74)
        da, db, dc = upload(api, a), upload(api, b), upload(api, c)
        api.check("sgemm", api.sgemm(h, op_a, op_b, m, n, k, 0.5, da, lda, db, ldb, 1.5, dc,
                                     ldc))
        out = np.empty_like(c)
        if op_a == 1 and op_b == 0:
            cuts = [0, 4 * (ldc * 333 + 5), 4 * (ldc * 2000 + 1), 4 * ldc * 3072, out.nbytes]
            for lo, hi in zip(cuts[:-1], cuts[1:]):
                api.d2h(ptr(out) + lo, dc + lo, hi - lo)
        else:
            api.d2h(ptr(out), dc, out.nbytes)
        key = f"{op_a}{op_b}m{math}"
        res["digests"][key] = hashlib.sha256(out.tobytes()).hexdigest()
        ref = oracle.gemm_sampled(op_a, op_b, k, 0.5, a, lda, b, ldb, 1.5, c, ldc, rows, cols,
                                  threads=16)
        o = out.reshape(n, ldc)
        res["errors"][key] = float(np.max(np.abs(o[cols, rows] - ref))) / k
        res["pad_kept"] = res.get("pad_kept", True) and bool(
            np.array_equal(o[:, m:], c.reshape(n, ldc)[:, m:]))
        for d in (da, db, dc):
            api.free(d)
    info = cp.runtime_info()
    res.update(deferred=info.gemm_deferred, blocks=info.gemm_column_blocks,
               in_place=info.gemm_in_place)
    res["shutdown"] = api.shutdown()
    return res


def scenario_deferred_evict(oracle):
    """Under a 512 MiB budget: a deferred GEMM whose C (128 MiB) is not read, then an
    8192 x 8192 x 4096 GEMM that streams and writes that C back to the host to free its
    frames, then C read (from the host copy) and updated in place by a second deferred
    GEMM, read in two pieces."""
    api = cp.CompatApi()
    init(api, cache_target=512 * MiB, chunk=64 * MiB)
    h = api.blas_create()
    m, n, k = 8192, 4096, 256
    a = oracle.uniform(m * k, 80).reshape(k, m)
    b = oracle.uniform(k * n, 81).reshape(n, k)
    c = oracle.uniform(m * n, 82).reshape(n, m)
    da, db, dc = upload(api, a), upload(api, b), upload(api, c)
    api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 0.5, da, m, db, k, 1.5, dc, m))
    bm, bn, bk = 8192, 8192, 4096
    x1 = oracle.uniform(bm * bk, 83)
    x2 = oracle.uniform(bk * bn, 84)
    d1, d2 = upload(api, x1), upload(api, x2)
    d3 = api.malloc(bm * bn * 4)
    api.check("sgemm", api.sgemm(h, 0, 0, bm, bn, bk, 1.0, d1, bm, d2, bk, 0.0, d3, bm))
    first = np.empty_like(c)
    api.d2h(ptr(first), dc, first.nbytes)
    rng = np.random.default_rng(6)
    rows, cols = rng.integers(0, m, 8192), rng.integers(0, n, 8192)
    ref = oracle.gemm_sampled(0, 0, k, 0.5, a, m, b, k, 1.5, c, m, rows, cols, threads=16)
    res = {"evicted_err": float(np.max(np.abs(first[cols, rows] - ref))) / k}
    api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 1.0, da, m, db, k, 1.0, dc, m))
    second = np.empty_like(c)
    half = 4 * (m * 1500 + 3)
    api.d2h(ptr(second), dc, half)
    api.d2h(ptr(second) + half, dc + half, second.nbytes - half)
    dot = oracle.gemm_sampled(0, 0, k, 1.0, a, m, b, k, 0.0, None, m, rows, cols, threads=16)
    res["second_err"] = float(np.max(np.abs(second[cols, rows] - (dot + first[cols, rows])))) / k
    t = api.telemetry()
    info = cp.runtime_info()
    res.update(dirty_evictions=t.runtime.dirty_evictions, streamed=info.gemm_streamed,
               deferred=info.gemm_deferred, blocks=info.gemm_column_blocks)
    res["shutdown"] = api.shutdown()
    return res


SCENARIOS = {name[len("scenario_"):]: fn for name, fn in globals().items()
             if name.startswith("scenario_")}

if __name__ == "__main__":
    result = SCENARIOS[sys.argv[1]](load_oracle())
    print(json.dumps(result, default=lambda o: o if not isinstance(o, tuple) else list(o)))
