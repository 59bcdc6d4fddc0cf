"""xvram_b200_sgemm_device_noalloc: the SGEMM entry point that allocates no device memory.

It is meant for callers that cannot allocate at the moment they run a GEMM (an application
whose allocator already owns all device memory, code inside that allocator's callbacks,
plugins limited to memory their host hands in).  Its scratch is a fixed array inside the
library, shared by every call.  These tests call it through the C ABI twice in a row on
different problems -- the second call finds the first call's leftovers in the array -- and
compare each result with the allocating entry point xvram_b200_sgemm_device, within the
tolerance the other parity tests use.  The file sorts last so that a run that stops at the
first failure has already run every other test; it also passes on its own.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle_lib import TOLERANCE, load_oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import device  # noqa: E402
from xvram_b200._native import lib  # noqa: E402

BUDGET_PRESSURE = 7
SCRATCH_BYTES = 32 << 20


def noalloc(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    stream = torch.cuda.current_stream().cuda_stream
    return lib.xvram_b200_sgemm_device_noalloc(op_a, op_b, m, n, k, alpha, A.data_ptr(), lda,
                                               B.data_ptr(), ldb, beta, C.data_ptr(), ldc, stream,
                                               0)


def problem(orc, op_a, op_b, m, n, k, seed):
    ra, ca = (k, m) if op_a else (m, k)
    rb, cb = (n, k) if op_b else (k, n)
    a = orc.uniform(ra * ca, seed).reshape(ca, ra)
    b = orc.uniform(rb * cb, seed + 1).reshape(cb, rb)
    c = orc.uniform(m * n, seed + 2).reshape(n, m)
    return a, ra, b, rb, c


def test_two_calls_in_a_row_match_the_allocating_entry_point():
    orc = load_oracle()
    cases = [(1, 0, 1000, 900, 1100, 0.5, 1.5, 70),   # TN: both operands transposed
             (0, 0, 777, 555, 333, -1.0, 0.25, 80)]   # NN: only B, fewer bytes than call 1
    for op_a, op_b, m, n, k, alpha, beta, seed in cases:
        need = device.workspace_bytes(op_a, op_b, m, n, k)
        assert 0 < need <= SCRATCH_BYTES
        a, lda, b, ldb, c = problem(orc, op_a, op_b, m, n, k, seed)
        A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        C_ref = torch.from_numpy(c).cuda()
        C_new = torch.from_numpy(c).cuda()
        assert device.sgemm(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, C_ref, m) == 0
        assert noalloc(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, C_new, m) == 0
        assert device.kernel_status() == 0
        want = C_ref.cpu().numpy().astype(np.float64)
        got = C_new.cpu().numpy().astype(np.float64)
        err = float(np.max(np.abs(got - want))) / (k * float(np.abs(a).max()) * float(np.abs(b).max()))
        assert err <= TOLERANCE, err


def test_problem_larger_than_the_scratch_array_is_refused():
    m, n, k = 4096, 4096, 2048       # TN needs 64 MiB of scratch, twice the array
    assert device.workspace_bytes(1, 0, m, n, k) > SCRATCH_BYTES
    A = torch.zeros((m, k), device="cuda")
    B = torch.zeros((n, k), device="cuda")
    C = torch.full((n, m), 3.0, device="cuda")
    assert noalloc(1, 0, m, n, k, 1.0, A, k, B, k, 0.0, C, m) == BUDGET_PRESSURE
    torch.cuda.synchronize()
    assert bool((C == 3.0).all())     # refused before anything was launched
