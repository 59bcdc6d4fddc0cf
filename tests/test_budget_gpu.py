"""Live device budget (reference src/residency/runtime.cpp:3213-3468): between operations
the runtime samples free device memory and shrinks its frame pool when another user takes
memory (writing dirty frames back first), then grows back once room returns."""
from __future__ import annotations

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import sdk  # noqa: E402

MiB = 1 << 20


def test_budget_shrinks_under_pressure_and_grows_back():
    import ctypes as C
    cfg = sdk.session_config(budget_poll_ms=1, device_headroom_bytes=1024 * MiB)
    with sdk.Sdk(cfg) as s:
        blocks = []
        for i in range(16):  # 4 GiB written straight to device frames (dirty)
            a = s.alloc(256 * MiB)
            a.write(np.full(64 * MiB, float(i + 1), dtype=np.float32))
            blocks.append(a)
        t0 = s.telemetry()

        def touch():  # any operation samples the budget first
            d = s.prefetch_desc([(blocks[0], 0, 4096, sdk.READ)])
            op = C.c_void_p()
            s.check("prefetch", s.t.prefetch_submit(s.session, C.byref(d), C.byref(op)))
            info = s.wait(op.value)
            s.t.operation_release(op.value)
            return info

        free, _ = torch.cuda.mem_get_info()
        hog = torch.empty(free - 256 * MiB, dtype=torch.uint8, device="cuda")
        time.sleep(0.01)
        assert touch().result == sdk.SUCCESS
        t1 = s.telemetry()
        assert t1.budget_shrinks >= 1
        assert t1.cache_target_bytes <= 4 * 1024 * MiB - 512 * MiB
        assert t1.dirty_evictions > t0.dirty_evictions       # written back before release
        assert t1.physical_handles_released > t0.physical_handles_released
        for i, a in enumerate(blocks):                         # nothing lost
            out = np.empty(64 * MiB, dtype=np.float32)
            a.read(out)
            assert out[0] == i + 1 and out[-1] == i + 1 and np.all(out[:: 1 << 20] == i + 1)
        del hog
        torch.cuda.empty_cache()
        # The sampler thread sees the freed memory within a few polls; the next operation
        # applies it.  Allow up to 2 s (a cold driver can answer the free-memory query late).
        deadline = time.monotonic() + 2.0
        while True:
            time.sleep(0.005)
            assert touch().result == sdk.SUCCESS
            t2 = s.telemetry()
            if t2.budget_grows >= 1 or time.monotonic() > deadline:
                break
        assert t2.budget_grows >= 1 and t2.cache_target_bytes > t1.cache_target_bytes
        assert t2.cache_target_minimum_bytes <= t1.cache_target_bytes
