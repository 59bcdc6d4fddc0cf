"""A kernel whose bounded pipeline wait runs out reports it through the kernels' error word;
the device entry point's status read returns it, the compat adapter turns it into TIMEOUT at
the next synchronising call and poisons itself, and the GPU stays usable.

The wait is made to run out with a hook of the test suite's own link of the library
(xvram_b200_test_set_kernel_stall, not exported by the product libraries): every CTA of
the FFMA kernel first waits on an mbarrier that nothing completes, for 2 ms, then takes
its abort path -- thread 0 waits for the TMA fills it already armed, every thread
returns.  Nothing faults, traps or hangs.  The reference's counterpart is its stall
timeout and poisoning (src/residency/runtime.cpp:3031-3051, docs/correctness.md:32-81).
The checks run in a child process bound to that link, so the product library loaded by
the rest of the suite is untouched.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

TESTS = Path(__file__).resolve().parent
ROOT = TESTS.parent

CHILD = r"""
import ctypes as C, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
import numpy as np, torch
from oracle_lib import TOLERANCE, load_oracle, normalized_error
from xvram_b200 import compat as cp, device as xd
from xvram_b200._native import lib
lib.xvram_b200_test_set_kernel_stall.argtypes = [C.c_ulonglong]
lib.xvram_b200_test_set_kernel_stall.restype = None
TIMEOUT, POISONED = 10, 15
orc = load_oracle()
m, n, k = 1024, 768, 512                      # op(A) = N, op(B) = T: no transposes
a, b, c = orc.uniform(m * k, 1), orc.uniform(n * k, 2), orc.uniform(m * n, 3)
A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()

# 1. the device entry point, for both tilings (1024 x 768 runs 128 x 256 tiles, 2304 x 2304
# runs 192 x 192): the launch succeeds, the error word says the wait ran out
for (mm, nn) in ((m, n), (2304, 2304)):
    aa, bb = orc.uniform(mm * k, 1), orc.uniform(nn * k, 2)
    AA, BB = torch.from_numpy(aa).cuda(), torch.from_numpy(bb).cuda()
    Cd = torch.zeros(mm * nn, device="cuda")
    lib.xvram_b200_test_set_kernel_stall(2_000_000)
    assert xd.sgemm(0, 1, mm, nn, k, 1.0, AA, mm, BB, nn, 0.0, Cd, mm, path=xd.PATH_TMA) == 0
    word = C.c_uint32(0)
    assert lib.xvram_b200_kernel_status(0, C.byref(word)) == 0
    assert word.value & 1, word.value             # bit 0: a consumer wait gave up
    assert xd.kernel_status() == 0                 # reading cleared it
    # the context is still usable: the same GEMM without the stall is correct
    lib.xvram_b200_test_set_kernel_stall(0)
    assert xd.sgemm(0, 1, mm, nn, k, 1.0, AA, mm, BB, nn, 0.0, Cd, mm, path=xd.PATH_TMA) == 0
    assert xd.kernel_status() == 0
    ref = orc.gemm(0, 1, mm, nn, k, 1.0, aa, mm, bb, nn, 0.0, None, mm)
    err = normalized_error(Cd.cpu().numpy().reshape(nn, mm), ref, k, 1.0, 1.0)
    assert err <= TOLERANCE, err
if torch.cuda.get_device_properties(0).multi_processor_count == 148:
    assert xd.tile_shape(m, n) == (128, 256) and xd.tile_shape(2304, 2304) == (192, 192)
Cd = torch.from_numpy(c).cuda()

# 2. the compat adapter: blas_sgemm returns once queued; the copy of C reports TIMEOUT
api = cp.CompatApi()
api.check("initialize", api.initialize())
h = api.blas_create()
ptrs = []
for arr in (a, b, c):
    d = api.malloc(arr.nbytes)
    api.h2d(d, arr.ctypes.data, arr.nbytes)
    ptrs.append(d)
lib.xvram_b200_test_set_kernel_stall(2_000_000)
st = api.sgemm(h, 0, 1, m, n, k, 1.0, ptrs[0], m, ptrs[1], n, 0.0, ptrs[2], m)
out = np.empty_like(c)
if st == 0:                                   # deferred: the next synchronising call reports it
    st = api.t.memcpy(out.ctypes.data, ptrs[2], out.nbytes, cp.D2H)
assert st == TIMEOUT, st
tel = api.telemetry()
assert tel.state == cp.STATE_POISONED, tel.state
assert api.t.memcpy(out.ctypes.data, ptrs[2], out.nbytes, cp.D2H) == POISONED
lib.xvram_b200_test_set_kernel_stall(0)
api.t.shutdown()
# the device is fine afterwards
assert xd.sgemm(0, 1, m, n, k, 1.0, A, m, B, n, 0.0, Cd, m, path=xd.PATH_TMA) == 0
assert xd.kernel_status() == 0
print("timeout path ok")
"""


def test_kernel_wait_that_runs_out_surfaces_as_timeout_and_poisons():
    from fake_device import testing_library
    lib = testing_library()
    env = dict(os.environ, XVRAM_B200_LIBRARY=str(lib))
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert "timeout path ok" in r.stdout
