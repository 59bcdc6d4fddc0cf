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


@pytest.mark.parametrize("op_a,op_b", [(1, 0), (0, 1)])
def test_three_k_chunks(oracle, op_a, op_b):
    """K = 5000 is three chunks of the tensor-core accumulation (three launches, each
    updating C in FP32 after the previous one)."""
    assert run(oracle, op_a, op_b, 1000, 777, 5000, 0.5, 1.5, seed=19) <= TOLERANCE


def test_long_k_accuracy(oracle):
    """K = 8192: the dropped lo*lo term and TF32 rounding of lo stay far below tolerance."""
    err = run(oracle, 1, 0, 256, 256, 8192, 1.0, 0.0, seed=13)
    assert err <= TOLERANCE / 10


def _positive_case(oracle, path, k):
    m, n = 256, 256
    a = (oracle.uniform(m * k, 21).reshape(m, k) + 1.0) * 0.5   # uniform[0, 1): same sign
    b = (oracle.uniform(k * n, 22).reshape(n, k) + 1.0) * 0.5
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    Cd = torch.zeros((n, m), device="cuda")
    assert device.sgemm(1, 0, m, n, k, 1.0, A, k, B, k, 0.0, Cd, m, path=path) == 0
    ref = oracle.gemm(1, 0, m, n, k, 1.0, a, k, b, k, 0.0, None, m, threads=16)
    out = Cd.cpu().numpy().astype(np.float64)
    return float(np.max(np.abs(out - ref) / np.abs(ref)))


@pytest.mark.parametrize("k", [512, 2048, 8192])
def test_same_sign_data_relative_error(oracle, k):
    """All-positive operands make the accumulator grow linearly, the worst case for the
    tensor core's FP32 accumulation.  The relative error must stay within the reference's
    own acceptance slope (2e-5 |ref|, src/compat_bench/executor.cpp:93-96) and within 8x
    the strict FFMA kernel's."""
    tc = _positive_case(oracle, TF32X3, k)
    ffma = _positive_case(oracle, 0, k)
    print(f"k={k} max relative error: tf32x3 {tc:.3e}  ffma {ffma:.3e}")
    assert tc <= 2e-5
    assert tc <= 8 * max(ffma, 2 ** -24)


def test_reference_gate_pattern_acceptance(oracle):
    """The reference's padded gate operands (compat_bench patterns, 37x19x67) through the
    tensor-core path meet the reference's own acceptance criterion."""
    import json
    from pathlib import Path
    from oracle_lib import reference_criterion
    g = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())
    fills = {(f["ta"], f["tb"], f["operand"]): f for f in g["cb_padded_fills"]["fills"]}
    shp = g["cb_padded_fills"]["shape"]
    m, n, k, off = shp["m"], shp["n"], shp["k"], shp["offset"]
    for ta in (0, 1):
        for tb in (0, 1):
            arrs = [np.frombuffer(bytes.fromhex(fills[(ta, tb, o)]["bits"]), np.float32).copy()
                    for o in range(3)]
            lds = [fills[(ta, tb, o)]["ld"] for o in range(3)]
            A, B, Cd = (torch.from_numpy(x).cuda() for x in arrs)
            st = device.sgemm(ta, tb, m, n, k, 0.5, A[off:], lds[0], B[off:], lds[1], 1.5,
                              Cd[off:], lds[2], path=TF32X3)
            assert st == 0
            out = Cd.cpu().numpy()
            ref = oracle.gemm(ta, tb, m, n, k, 0.5, arrs[0][off:], lds[0], arrs[1][off:], lds[1],
                              1.5, arrs[2][off:], lds[2])
            body = np.stack([out[off + j * lds[2]: off + j * lds[2] + m] for j in range(n)])
            assert reference_criterion(body, ref)
