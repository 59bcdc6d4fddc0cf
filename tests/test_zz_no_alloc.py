"""xvram_b200_sgemm_device_noalloc: the SGEMM entry point that allocates no device memory.

It is meant for callers that cannot allocate at the moment they run a GEMM (an application
whose allocator already owns all device memory, code inside that allocator's callbacks,
plugins limited to memory their host hands in).  Its scratch is a fixed array inside the
library, shared by every call.  These tests call it through the C ABI twice in a row on
different problems -- the second call finds the first call's leftovers in the array -- and
require each result to be bit-identical to the allocating entry point
xvram_b200_sgemm_device (both run the same transposes and kernel) and within the SGEMM
tolerance of the CPU FP64 oracle.  After the first call, a further call must not change
the device's free memory.  The file sorts last so that a run that stops at the first
failure has already run every other test; it also passes on its own.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle_lib import TOLERANCE, load_oracle, normalized_error

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import device  # noqa: E402
from xvram_b200._native import lib  # noqa: E402

INVALID_ARGUMENT = 1
BUDGET_PRESSURE = 7
SCRATCH_BYTES = 32 << 20
PATH_TF32X3 = 3


def noalloc(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, path=0) -> int:
    stream = torch.cuda.current_stream().cuda_stream
    return lib.xvram_b200_sgemm_device_noalloc(op_a, op_b, m, n, k, alpha, A.data_ptr(), lda,
                                               B.data_ptr(), ldb, beta, C.data_ptr(), ldc, stream,
                                               path)


def problem(orc, op_a, op_b, m, n, k, seed):
    ra, ca = (k, m) if op_a else (m, k)
    rb, cb = (n, k) if op_b else (k, n)
    a = orc.uniform(ra * ca, seed).reshape(ca, ra)
    b = orc.uniform(rb * cb, seed + 1).reshape(cb, rb)
    c = orc.uniform(m * n, seed + 2).reshape(n, m)
    return a, ra, b, rb, c


def test_two_calls_in_a_row_match_the_allocating_entry_point_and_the_oracle():
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
        want = C_ref.cpu().numpy()
        got = C_new.cpu().numpy()
        # Same transposes, same kernel: the results agree bit for bit.
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        ref = orc.gemm(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, m)
        err = normalized_error(got, ref, k, float(np.abs(a).max()), float(np.abs(b).max()))
        assert err <= TOLERANCE, err


def test_a_call_after_the_first_takes_no_device_memory():
    orc = load_oracle()
    m, n, k = 1024, 768, 1536                       # TN: 10.5 MiB of scratch
    a, lda, b, ldb, c = problem(orc, 1, 0, m, n, k, 90)
    A, B, C = (torch.from_numpy(x).cuda() for x in (a, b, c))
    assert noalloc(1, 0, m, n, k, 1.0, A, lda, B, ldb, 0.0, C, m) == 0   # first call: loads
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert noalloc(1, 0, m, n, k, 1.0, A, lda, B, ldb, 0.5, C, m) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert device.kernel_status() == 0


def test_tensor_core_path_is_not_offered():
    A = torch.zeros((64, 64), device="cuda")
    C = torch.full((64, 64), 2.0, device="cuda")
    assert noalloc(0, 0, 64, 64, 64, 1.0, A, 64, A, 64, 0.0, C, 64, path=PATH_TF32X3) == \
        INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert bool((C == 2.0).all())


def test_problem_larger_than_the_scratch_array_is_refused():
    m, n, k = 4096, 4096, 2048       # TN needs 64 MiB of scratch, twice the array
    assert device.workspace_bytes(1, 0, m, n, k) > SCRATCH_BYTES
    A = torch.zeros((m, k), device="cuda")
    B = torch.zeros((n, k), device="cuda")
    C = torch.full((n, m), 3.0, device="cuda")
    assert noalloc(1, 0, m, n, k, 1.0, A, k, B, k, 0.0, C, m) == BUDGET_PRESSURE
    torch.cuda.synchronize()
    assert bool((C == 3.0).all())     # refused before anything was launched
