"""Tensor-core FP32 path (3xTF32 on tcgen05/TMEM) against the CPU FP64 oracle.

The path is FP32-accurate, not bit-identical to the FFMA kernels: each operand is split
into TF32 hi + lo parts and three TF32 products are accumulated in FP32.  It must meet the
same stated tolerance as every other path: max|err| / (K max|a| max|b|) <= 1e-6."""
from __future__ import annotations

import numpy as np
import pytest

from oracle_lib import TOLERANCE, normalized_error

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import device  # noqa: E402
from xvram_b200._native import lib  # noqa: E402

TF32X3 = 3
WS_TF32X3 = 0x100


def run(oracle, op_a, op_b, m, n, k, alpha, beta, seed=0, pad=(0, 0, 0), explicit_ws=False):
    ra, ca = (k, m) if op_a else (m, k)
    rb, cb = (n, k) if op_b else (k, n)
    lda, ldb, ldc = ra + pad[0], rb + pad[1], m + pad[2]
    a = oracle.uniform(ca * lda, seed).reshape(ca, lda)
    b = oracle.uniform(cb * ldb, seed + 1).reshape(cb, ldb)
    c = oracle.uniform(n * ldc, seed + 2).reshape(n, ldc)
    A, B, Cd = (torch.from_numpy(x).cuda() for x in (a, b, c))
    if explicit_ws:
        need = lib.xvram_b200_sgemm_workspace_bytes(op_a | WS_TF32X3, op_b, m, n, k)
        ws = torch.empty(need // 4 + 64, device="cuda")
        st = device.sgemm_ws(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, Cd, ldc, ws, need,
                             path=TF32X3)
    else:
        st = device.sgemm(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, Cd, ldc, path=TF32X3)
    assert st == 0
    assert device.kernel_status() == 0
    out = Cd.cpu().numpy()
    ref = oracle.gemm(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, None if beta == 0 else c,
                      ldc, threads=16)
    err = normalized_error(out[:, :m], ref, k, float(np.abs(a).max()), float(np.abs(b).max()))
    assert np.array_equal(out[:, m:], c[:, m:])
    return err


def test_single_tile(oracle):
    assert run(oracle, 1, 0, 128, 256, 16, 1.0, 0.0) <= TOLERANCE


@pytest.mark.parametrize("op_a,op_b", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("shape", [(300, 200, 100), (1000, 777, 513), (129, 257, 1)])
def test_ragged_shapes_all_operations(oracle, op_a, op_b, shape):
    m, n, k = shape
    assert run(oracle, op_a, op_b, m, n, k, 0.5, 1.5, seed=7, pad=(3, 2, 1)) <= TOLERANCE


def test_explicit_workspace_and_beta_zero(oracle):
    assert run(oracle, 0, 1, 700, 600, 900, -1.25, 0.0, seed=11, explicit_ws=True) <= TOLERANCE


def test_long_k_accuracy(oracle):
    """K = 8192: the dropped lo*lo term and TF32 rounding of lo stay far below tolerance."""
    err = run(oracle, 1, 0, 256, 256, 8192, 1.0, 0.0, seed=13)
    assert err <= TOLERANCE / 10
