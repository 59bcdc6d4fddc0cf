"""FP16 / BF16 / FP64 GEMMs on the B200 against the CPU oracle: the device entry point
(widening pass + FFMA kernel; FP64 tensor-core kernel) over every operation pair and
ragged shapes, C = beta C for k = 0, long-K FP64 accuracy, and the SDK plan API in place
and out of core (FP16 C accumulated in FP32 in its slot).  Tolerances in typed_util."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from typed_util import (BF16, FP16, FP32, FP64, FP64_TOLERANCE, check, decode, make_problem,
                        reference)

from xvram_b200 import device as xd
from xvram_b200 import sdk

pytestmark = pytest.mark.gpu
MiB = 1 << 20
TORCH = {FP16: torch.float16, BF16: torch.bfloat16, FP32: torch.float32, FP64: torch.float64}


def to_device(stored: np.ndarray, dtype: int) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(stored))
    if dtype in (FP16, BF16):
        t = t.view(torch.int16).view(TORCH[dtype])
    return t.cuda()


def from_device(t: torch.Tensor, dtype: int) -> np.ndarray:
    t = t.cpu()
    if dtype in (FP16, BF16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def run_device(ab, ct, op_a, op_b, m, n, k, alpha, beta, seed, pad=0):
    A, B, Cs, av, bv, cv = make_problem(ab, ct, op_a, op_b, m, n, k, seed)
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    Ad, Bd = to_device(A, ab), to_device(B, ab)
    Cd = to_device(Cs, ct)
    assert xd.gemm_typed(op_a, op_b, m, n, k, alpha, Ad, lda, Bd, ldb, beta, Cd, m) == 0
    torch.cuda.synchronize()
    out = from_device(Cd, ct)
    ref = reference(ab, op_a, op_b, m, n, k, alpha, av, bv, beta, cv)
    return check(ab, ct, out, ref, max(k, 1))


COMBOS = [(FP16, FP16), (FP16, FP32), (BF16, BF16), (BF16, FP32), (FP64, FP64)]


@pytest.mark.parametrize("ab,ct", COMBOS)
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("shape", [(300, 200, 100), (129, 257, 33), (1, 1, 1), (515, 389, 611)])
def test_device_typed_gemm_matches_oracle(ab, ct, op_a, op_b, shape):
    m, n, k = shape
    run_device(ab, ct, op_a, op_b, m, n, k, 0.75, -1.25, 7)


@pytest.mark.parametrize("ab,ct", COMBOS)
def test_beta_zero_never_reads_c(ab, ct):
    """beta == 0: C's previous contents (here NaN) are not read."""
    m, n, k = 200, 150, 90
    A, B, Cs, av, bv, _ = make_problem(ab, ct, 0, 0, m, n, k, 3)
    Cd = torch.full((n, m), float("nan"), dtype=TORCH[ct], device="cuda")
    assert xd.gemm_typed(0, 0, m, n, k, 1.0, to_device(A, ab), m, to_device(B, ab), k, 0.0, Cd,
                         m) == 0
    out = from_device(Cd, ct)
    assert np.isfinite(decode(out, ct)).all()
    check(ab, ct, out, reference(ab, 0, 0, m, n, k, 1.0, av, bv, 0.0, None), k)


def test_fp64_long_k_accuracy():
    """K = 8192 in FP64: far below the FP64 bound, and far below what FP32 arithmetic on
    the same data would give (~1e-8)."""
    err = run_device(FP64, FP64, 1, 0, 256, 256, 8192, 1.0, 0.0, 13)
    assert err <= FP64_TOLERANCE / 100


def test_fp16_products_are_exact_in_fp32():
    """FP16 inputs under strict FP32 arithmetic: the result equals the FP32 FFMA kernel
    run on the widened values, bit for bit (widening and FP16 x FP16 products are exact)."""
    m, n, k = 384, 256, 320
    A, B, Cs, av, bv, cv = make_problem(FP16, FP32, 1, 0, m, n, k, 17)
    Cd = to_device(Cs, FP32)
    assert xd.gemm_typed(1, 0, m, n, k, 0.5, to_device(A, FP16), k, to_device(B, FP16), k, 1.5,
                         Cd, m) == 0
    A32 = torch.from_numpy(av.astype(np.float32)).cuda()
    B32 = torch.from_numpy(bv.astype(np.float32)).cuda()
    C32 = to_device(Cs, FP32)
    assert xd.sgemm(1, 0, m, n, k, 0.5, A32, k, B32, k, 1.5, C32, m) == 0
    torch.cuda.synchronize()
    assert torch.equal(Cd, C32)


def sdk_run(s, ab, ct, op_a, op_b, m, n, k, alpha, beta, seed):
    A, B, Cs, av, bv, cv = make_problem(ab, ct, op_a, op_b, m, n, k, seed)
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    allocs = []
    for arr in (A, B, Cs):
        h = s.alloc(arr.nbytes)
        h.write(np.ascontiguousarray(arr))
        allocs.append(h)
    Ad, Bd, Cd = allocs
    desc = s.gemm_desc(sdk.matrix(Ad, m if op_a == 0 else k, k if op_a == 0 else m, lda,
                                  data_type=ab),
                       sdk.matrix(Bd, k if op_b == 0 else n, n if op_b == 0 else k, ldb,
                                  data_type=ab),
                       sdk.matrix(Cd, m, n, m, data_type=ct), op_a, op_b, alpha=alpha,
                       beta=beta)
    plan = s.plan(desc)
    info = s.plan_info(plan)
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    out = np.empty_like(Cs)
    Cd.read(out)
    check(ab, ct, out, reference(ab, op_a, op_b, m, n, k, alpha, av, bv, beta, cv), k)
    return info


@pytest.mark.parametrize("ab,ct", COMBOS)
def test_sdk_typed_plans_in_place(ab, ct):
    with sdk.Sdk(sdk.session_config()) as s:
        info = sdk_run(s, ab, ct, 1, 0, 700, 520, 300, 0.5, 1.5, 21)
        assert info.tile_count == 1
        want = sdk.COMPUTE_FP64 if ab == FP64 else sdk.COMPUTE_FP32_STRICT
        assert info.effective_compute_mode == want


@pytest.mark.parametrize("ab,ct,beta", [(FP16, FP16, 1.0), (BF16, FP32, 0.5),
                                        (FP64, FP64, 1.0)])
def test_sdk_typed_plans_out_of_core(ab, ct, beta):
    """Operands above a 16 MiB budget of 2 MiB frames: the panel schedule with element
    sizes 2 and 8 (and an FP16 C accumulated in FP32 in its slot) gives the in-place
    numbers."""
    m, n, k = (2048, 1536, 1536) if ab != FP64 else (1024, 768, 768)
    if ct == FP32:
        m, n, k = 1536, 1536, 1536
    cfg = sdk.session_config(chunk_size_bytes=2 * MiB, cache_target_bytes=16 * MiB)
    with sdk.Sdk(cfg) as s:
        info = sdk_run(s, ab, ct, 0, 1, m, n, k, 1.0, beta, 29)
        assert info.tile_count > 1 and info.maximum_working_set_bytes <= 16 * MiB
        tel = s.telemetry()
        assert tel.handle_reuses > 0 and tel.resident_bytes_peak <= 16 * MiB
