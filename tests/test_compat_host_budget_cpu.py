"""Host-memory admission of the compat adapter (reference
src/cuda_compat/runtime_backend.cpp:103-139), on the host-memory fake device.

At initialisation the adapter reads the host's physical and available RAM, keeps
max(4 GiB, physical / 4) of it free (host_headroom_bytes) and caps the runtime's host
ledger -- the pinned host backing of allocations -- at the rest (host_store_cap_bytes).
The telemetry reports both, and host_budget_bytes follows the ledger: the backing that
allocations whose chunks left the device hold, zero after shutdown.  Runs in a child
process (one compat initialisation per process)."""
from __future__ import annotations

import json
import subprocess
import sys

from fake_device import ROOT

SCRIPT = r"""
import json, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
import numpy as np
from fake_device import installed
from xvram_b200 import compat as cp
with installed():
    api = cp.CompatApi()
    cfg = cp.compat_config_init()
    cfg.session.chunk_size_bytes = 2 << 20
    cfg.session.cache_target_bytes = 64 << 20
    api.check("initialize", api.initialize(cfg))
    t0 = api.telemetry()
    x = np.ones(12 << 20, dtype=np.float32)          # 48 MiB, twice: above the 64 MiB cache
    ps = [api.malloc(x.nbytes) for _ in range(2)]
    for p in ps:
        api.h2d(p, x.ctypes.data, x.nbytes)
    t1 = api.telemetry()
    for p in ps:
        api.free(p)
    api.t.shutdown()
    out = cp.CompatTelemetry()
    import ctypes as C
    out.struct_size = C.sizeof(cp.CompatTelemetry)
    api.t.get_telemetry(C.byref(out))
    pick = lambda t: {f: int(getattr(t, f)) for f in (
        "host_physical_bytes", "host_available_bytes", "host_store_cap_bytes",
        "host_headroom_bytes", "host_budget_bytes", "host_backing_bytes",
        "retired_va_reservations", "retired_va_reservations_freed")}
    print(json.dumps([pick(t0), pick(t1), pick(out)]))
"""


def test_host_headroom_cap_and_ledger():
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    t0, t1, fin = json.loads(r.stdout.strip().splitlines()[-1])
    phys, avail = t0["host_physical_bytes"], t0["host_available_bytes"]
    assert phys > 0 and 0 < avail <= phys
    assert t0["host_headroom_bytes"] == max(4 << 30, phys // 4)
    assert t0["host_store_cap_bytes"] == avail - t0["host_headroom_bytes"]
    assert t0["host_budget_bytes"] == 0
    # 96 MiB through a 64 MiB cache: evicted chunks live in host backing
    assert t1["host_budget_bytes"] == t1["host_backing_bytes"] >= 48 << 20
    assert t1["host_budget_bytes"] <= t1["host_store_cap_bytes"]
    # after shutdown: the ledger is empty, the freed range's reservation was released
    assert fin["host_budget_bytes"] == 0
    assert fin["retired_va_reservations"] == 0 and fin["retired_va_reservations_freed"] == 2
