"""Deferred completion of the compat blas_sgemm on the host-memory fake device.

By default blas_sgemm returns once its kernels are queued, as cublasSgemm does: an
in-place strict-FP32 GEMM runs as column blocks of C, and the next cudaMemcpy of C copies
each block after its own kernel.  These tests drive that path with a fake that reports 2
SMs (so small problems split into several blocks):
  * every operation, with ldc > m, matches the oracle and is bit-identical to the
    synchronous call (XVRAM_B200_SYNC_GEMM=1, the reference's completion rule);
  * reads of C in pieces that start and end inside blocks return the same bytes;
  * a kernel error word found after the call fails the next memcpy with TIMEOUT and
    poisons the adapter (the sticky-error rule of the asynchronous call);
  * freeing C without reading it, and cudaDeviceSynchronize, leave the adapter ready.
Each scenario runs in a child process (one compat initialisation per process)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from oracle_lib import TOLERANCE

SCRIPT = r"""
import hashlib, json, sys
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
from fake_device import installed
from oracle_lib import load_oracle, normalized_error
from xvram_b200 import compat as cp

mode = sys.argv[2]
with installed() as fake:
    fake.fake_device_set_sm_count(2)
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.chunk_size_bytes = 2 << 20
    cfg.session.cache_target_bytes = 64 << 20
    api.check("initialize", api.initialize(cfg))
    orc = load_oracle()
    h = api.blas_create()
    m, n, k = 500, 1800, 96
    if mode == "narrow":
        n = 2800  # 11 tile columns in 8 blocks: one-column first and last blocks
    ldc = m + 6
    out = {"results": {}, "errors": {}}
    if mode in ("ops", "tf32", "narrow"):
        if mode == "tf32":  # math mode 3; the fake computes it in strict FP32
            api.check("math", api.t.blas_set_math_mode(h, 3))
        p0 = fake.fake_device_prepares()
        for op_a in (0, 1):
            for op_b in (0, 1):
                if mode == "narrow" and (op_a, op_b) != (1, 0):
                    continue
                lda = m if op_a == 0 else k
                ldb = k if op_b == 0 else n
                a = orc.uniform(lda * (k if op_a == 0 else m), 10 + op_a)
                b = orc.uniform(ldb * (n if op_b == 0 else k), 20 + op_b)
                c = orc.uniform(ldc * n, 30)
                pa, pb, pc = (api.malloc(x.nbytes) for x in (a, b, c))
                for p, x in zip((pa, pb, pc), (a, b, c)):
                    api.h2d(p, x.ctypes.data, x.nbytes)
                api.check("sgemm", api.sgemm(h, op_a, op_b, m, n, k, 0.5, pa, lda, pb, ldb, 1.5,
                                             pc, ldc))
                got = np.empty(ldc * n, np.float32)
                if op_a == 1 and op_b == 0:  # in pieces that cut through blocks
                    cuts = [0, 4 * (ldc * 100 + 7), 4 * (ldc * 700 + 3), 4 * ldc * 1024, got.nbytes]
                    for lo, hi in zip(cuts[:-1], cuts[1:]):
                        api.d2h(got.ctypes.data + lo, pc + lo, hi - lo)
                else:
                    api.d2h(got.ctypes.data, pc, got.nbytes)
                ref = orc.gemm(op_a, op_b, m, n, k, 0.5, a, lda, b, ldb, 1.5, c, ldc)
                g = got.reshape(n, ldc)[:, :m]
                err = normalized_error(g, ref, k, 1.0, 1.0)  # ref is (n, m)
                pad_kept = bool(np.array_equal(got.reshape(n, ldc)[:, m:], c.reshape(n, ldc)[:, m:]))
                out["results"][f"{op_a}{op_b}"] = {"err": float(err), "pad_kept": pad_kept,
                                                   "digest": hashlib.sha256(got.tobytes()).hexdigest()}
                for p in (pa, pb, pc):
                    api.free(p)
        out["prepares"] = int(fake.fake_device_prepares() - p0)
    elif mode == "evict":
        # a deferred GEMM whose C is not read, then a GEMM too large for the 64 MiB budget
        # (streamed: it writes the first C back to the host to free its frames), then C
        # written again by a third, in-place GEMM whose result is read in pieces
        a, b, c = orc.uniform(m * k, 1), orc.uniform(k * n, 2), orc.uniform(ldc * n, 3)
        pa, pb, pc = (api.malloc(x.nbytes) for x in (a, b, c))
        for p, x in zip((pa, pb, pc), (a, b, c)):
            api.h2d(p, x.ctypes.data, x.nbytes)
        api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 0.5, pa, m, pb, k, 1.5, pc, ldc))
        big = 2816
        x1, x2 = orc.uniform(big * big, 4), orc.uniform(big * big, 5)
        p1, p2, p3 = (api.malloc(big * big * 4) for _ in range(3))
        api.h2d(p1, x1.ctypes.data, x1.nbytes)
        api.h2d(p2, x2.ctypes.data, x2.nbytes)
        api.check("sgemm", api.sgemm(h, 0, 0, big, big, big, 1.0, p1, big, p2, big, 0.0, p3, big))
        got = np.empty(ldc * n, np.float32)
        api.d2h(got.ctypes.data, pc, got.nbytes)
        ref = orc.gemm(0, 0, m, n, k, 0.5, a, m, b, k, 1.5, c, ldc)
        out["evicted_err"] = float(normalized_error(got.reshape(n, ldc)[:, :m], ref, k, 1.0, 1.0))
        # C holds the first result; a second deferred GEMM updates it in place again
        api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 1.0, pa, m, pb, k, 1.0, pc, ldc))
        got2 = np.empty_like(got)
        half = 4 * (ldc * 901 + 11)
        api.d2h(got2.ctypes.data, pc, half)
        api.d2h(got2.ctypes.data + half, pc + half, got2.nbytes - half)
        dot = orc.gemm(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
        out["second_err"] = float(normalized_error(got2.reshape(n, ldc)[:, :m],
                                                   dot + got.reshape(n, ldc)[:, :m], k, 1.0, 1.0))
        tel = api.telemetry()
        out["dirty_evictions"] = int(tel.runtime.dirty_evictions)
        out["streamed"] = int(cp.runtime_info().gemm_streamed)
    elif mode == "misc":
        # (1) C inside a larger allocation, after 3 MiB of other data: a read of the whole
        # allocation mixes bytes outside the column blocks with the blocks themselves;
        # (2) A and B freed before C is read; (3) a GEMM below two waves of tiles runs
        # whole (no column blocks) but still returns before its kernel.
        a, b = orc.uniform(m * k, 1), orc.uniform(k * n, 2)
        c = orc.uniform(ldc * n, 3)
        lead = orc.uniform(3 * 262144, 4)                     # 3 MiB before C
        pa, pb = (api.malloc(x.nbytes) for x in (a, b))
        pbig = api.malloc(lead.nbytes + c.nbytes + 4096)
        api.h2d(pa, a.ctypes.data, a.nbytes)
        api.h2d(pb, b.ctypes.data, b.nbytes)
        api.h2d(pbig, lead.ctypes.data, lead.nbytes)
        api.h2d(pbig + lead.nbytes, c.ctypes.data, c.nbytes)
        pc = pbig + lead.nbytes
        api.check("sgemm", api.sgemm(h, 0, 0, m, n, k, 0.5, pa, m, pb, k, 1.5, pc, ldc))
        api.free(pa)
        api.free(pb)
        whole = np.empty((lead.nbytes + c.nbytes) // 4, np.float32)
        api.d2h(whole.ctypes.data, pbig, whole.nbytes)
        got = whole[lead.size:]
        ref = orc.gemm(0, 0, m, n, k, 0.5, a, m, b, k, 1.5, c, ldc)
        out["misc_err"] = float(normalized_error(got.reshape(n, ldc)[:, :m], ref, k, 1.0, 1.0))
        out["lead_kept"] = bool(np.array_equal(whole[:lead.size], lead))
        blocks_before = int(cp.runtime_info().gemm_column_blocks)
        sm, sn, sk = 128, 256, 64                            # one tile: launched whole
        x, y = orc.uniform(sm * sk, 5), orc.uniform(sk * sn, 6)
        px, py, pz = api.malloc(x.nbytes), api.malloc(y.nbytes), api.malloc(sm * sn * 4)
        api.h2d(px, x.ctypes.data, x.nbytes)
        api.h2d(py, y.ctypes.data, y.nbytes)
        api.check("sgemm", api.sgemm(h, 0, 0, sm, sn, sk, 1.0, px, sm, py, sk, 0.0, pz, sm))
        z = np.empty(sm * sn, np.float32)
        api.d2h(z.ctypes.data, pz, z.nbytes)
        zref = orc.gemm(0, 0, sm, sn, sk, 1.0, x, sm, y, sk, 0.0, None, sm)
        out["small_err"] = float(normalized_error(z.reshape(sn, sm), zref, sk, 1.0, 1.0))
        out["small_blocks"] = int(cp.runtime_info().gemm_column_blocks) - blocks_before
    elif mode == "error":
        a, b, c = orc.uniform(m * k, 1), orc.uniform(k * n, 2), orc.uniform(ldc * n, 3)
        pa, pb, pc = (api.malloc(x.nbytes) for x in (a, b, c))
        for p, x in zip((pa, pb, pc), (a, b, c)):
            api.h2d(p, x.ctypes.data, x.nbytes)
        # a GEMM whose C is freed unread, then a synchronize: both fine
        pc2 = api.malloc(c.nbytes)
        api.h2d(pc2, c.ctypes.data, c.nbytes)
        out["errors"]["sgemm_unread"] = api.sgemm(h, 0, 0, m, n, k, 1.0, pa, m, pb, k, 0.0, pc2, ldc)
        out["errors"]["free_unread"] = api.t.free_device(pc2)
        out["errors"]["synchronize"] = api.t.synchronize()
        out["errors"]["sgemm"] = api.sgemm(h, 0, 0, m, n, k, 1.0, pa, m, pb, k, 0.0, pc, ldc)
        fake.fake_device_set_kernel_word(1)  # the queued kernels' bounded wait ran out
        got = np.empty(ldc * n, np.float32)
        out["errors"]["d2h"] = api.t.memcpy(got.ctypes.data, pc, got.nbytes, cp.D2H)
        out["errors"]["after"] = api.t.memcpy(got.ctypes.data, pc, got.nbytes, cp.D2H)
        out["state"] = api.telemetry().state
    info = cp.runtime_info()
    out["deferred"] = int(info.gemm_deferred)
    out["blocks"] = int(info.gemm_column_blocks)
    out["in_place"] = int(info.gemm_in_place)
    out["shutdown"] = api.shutdown()
    print(json.dumps(out))
"""


def run(mode: str, sync: bool = False) -> dict:
    from fake_device import ROOT
    env = dict(os.environ)
    env.pop("XVRAM_B200_SYNC_GEMM", None)
    if sync:
        env["XVRAM_B200_SYNC_GEMM"] = "1"
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), mode], capture_output=True,
                       text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_column_blocks_match_the_oracle_and_the_synchronous_call():
    deferred = run("ops")
    sync = run("ops", sync=True)
    # 4 tiles of 128 rows x 8 of 256 columns on 2 SMs: 8 blocks of 256 columns each
    assert deferred["in_place"] == 4 and deferred["deferred"] == 4
    assert deferred["blocks"] == 4 * 8
    assert sync["deferred"] == 0 and sync["blocks"] == 0
    # the operands are prepared once per call, not once per block
    assert deferred["prepares"] == 4 and sync["prepares"] == 0
    for key, r in deferred["results"].items():
        assert r["err"] <= TOLERANCE, key
        assert r["pad_kept"], key  # rows m..ldc of C are not written
        assert r["digest"] == sync["results"][key]["digest"], key  # bit-identical
    assert deferred["shutdown"] == 0 and sync["shutdown"] == 0


def test_tensor_core_mode_splits_by_tile_pairs():
    """Math mode 3: tiles are 256 x 256 on SM pairs, so with 2 SMs (one pair) the 2 x 8
    tiles make 8 blocks as well."""
    d = run("tf32")
    s = run("tf32", sync=True)
    assert d["deferred"] == 4 and d["blocks"] == 4 * 8 and d["prepares"] == 4
    for key, r in d["results"].items():
        assert r["err"] <= TOLERANCE and r["pad_kept"], key
        assert r["digest"] == s["results"][key]["digest"], key


def test_kernel_error_surfaces_at_the_next_copy():
    r = run("error")
    e = r["errors"]
    assert e["sgemm_unread"] == 0 and e["free_unread"] == 0 and e["synchronize"] == 0
    assert e["sgemm"] == 0
    assert e["d2h"] == 10            # XVRAM_STATUS_TIMEOUT
    assert e["after"] == 15          # XVRAM_STATUS_POISONED
    assert r["state"] == 3           # XVRAM_CUDA_COMPAT_POISONED
    assert r["deferred"] == 2


def test_deferred_result_survives_eviction_by_a_streamed_gemm():
    """A deferred GEMM's C, never read, is written back to the host when a larger,
    streamed GEMM needs its frames; reading it afterwards (from the host copy) and updating
    it with another deferred GEMM both give the right values."""
    r = run("evict")
    assert r["streamed"] == 1 and r["dirty_evictions"] > 0
    assert r["evicted_err"] <= TOLERANCE and r["second_err"] <= TOLERANCE
    assert r["deferred"] == 2 and r["shutdown"] == 0


def test_narrow_first_and_last_blocks():
    """11 tile columns in 8 blocks: the first and last are one tile column wide, the six
    between share the other nine; the result is still bit-identical."""
    d = run("narrow")
    s = run("narrow", sync=True)
    assert d["deferred"] == 1 and d["blocks"] == 8
    r = d["results"]["10"]
    assert r["err"] <= TOLERANCE and r["pad_kept"]
    assert r["digest"] == s["results"]["10"]["digest"]


def test_c_inside_a_larger_allocation_and_operands_freed_early():
    """C at a 3 MiB offset of a larger allocation, A and B freed before C is read, the whole
    allocation read at once (bytes outside the column blocks and the blocks together);
    and a one-tile GEMM, which runs whole but still returns before its kernel."""
    r = run("misc")
    assert r["misc_err"] <= TOLERANCE and r["lead_kept"]
    assert r["small_err"] <= TOLERANCE and r["small_blocks"] == 0
    assert r["deferred"] == 2 and r["shutdown"] == 0
