"""FP16 / BF16 / FP64 GEMMs through the SDK on the host-memory fake device: plan
validation and the compute-mode mapping of the reference (src/sdk/runtime.cpp:119-142,
src/gemm/planner.cpp:819-842), the typed in-place path, and the out-of-core panel replay
with element sizes other than 4 -- including an FP16 / BF16 C that accumulates in FP32 in
its slot and is converted on the way in and out.  The fake's GEMM is a plain loop (FP32
fmaf for FP32 arithmetic, FP64 fma for FP64)."""
from __future__ import annotations

import numpy as np
import pytest

from fake_device import installed
from typed_util import BF16, ESIZE, FP16, FP32, FP64, check, make_problem, reference

from xvram_b200 import sdk

MiB = 1 << 20


def session(budget=0, chunk=2 * MiB):
    return sdk.Sdk(sdk.session_config(cache_target_bytes=budget, chunk_size_bytes=chunk))


def upload(s, arr):
    a = s.alloc(max(arr.nbytes, 1))
    a.write(np.ascontiguousarray(arr))
    return a


def run(s, ab, ct, op_a, op_b, m, n, k, alpha, beta, seed, mode=sdk.COMPUTE_AUTO):
    A, B, Cs, av, bv, cv = make_problem(ab, ct, op_a, op_b, m, n, k, seed)
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    Ad, Bd, Cd = upload(s, A), upload(s, B), upload(s, Cs)
    desc = s.gemm_desc(sdk.matrix(Ad, m if op_a == 0 else k, k if op_a == 0 else m, lda,
                                  data_type=ab),
                       sdk.matrix(Bd, k if op_b == 0 else n, n if op_b == 0 else k, ldb,
                                  data_type=ab),
                       sdk.matrix(Cd, m, n, m, data_type=ct), op_a, op_b, alpha=alpha,
                       beta=beta, mode=mode)
    plan = s.plan(desc)
    info = s.plan_info(plan)
    s.check("gemm_execute", s.t.gemm_execute(plan, sdk.TIMEOUT_INFINITE))
    s.t.gemm_plan_release(plan)
    out = np.empty_like(Cs)
    Cd.read(out)
    ref = reference(ab, op_a, op_b, m, n, k, alpha, av, bv, beta, cv)
    return check(ab, ct, out, ref, k), info


COMBOS = [(FP16, FP16), (FP16, FP32), (BF16, BF16), (BF16, FP32), (FP64, FP64)]


@pytest.mark.parametrize("ab,ct", COMBOS)
@pytest.mark.parametrize("op_a,op_b", [(0, 0), (1, 0), (0, 1)])
def test_typed_in_place(ab, ct, op_a, op_b):
    with installed(), session() as s:
        _, info = run(s, ab, ct, op_a, op_b, 70, 45, 33, 0.5, 1.5, 5)
        assert info.tile_count == 1
        want = {FP64: sdk.COMPUTE_FP64}.get(ab, sdk.COMPUTE_FP32_STRICT)
        assert info.effective_compute_mode == want


@pytest.mark.parametrize("ab,ct,beta", [(FP16, FP16, 1.0), (BF16, FP32, 1.0),
                                        (FP64, FP64, 0.5), (BF16, BF16, 0.0)])
def test_typed_streamed_under_a_small_budget(ab, ct, beta):
    """Operands above a 16 MiB budget: a streamed panel schedule with evictions,
    element sizes 2 and 8, and for a half C the FP32 accumulation slot with its staging
    copy."""
    m, n, k = 2048, 1536, 1536       # FP16 / BF16: 16.5 MiB with a 2-byte C
    if ct == FP32:
        m, n, k = 1536, 1536, 1536   # 4.5 + 4.5 + 9 MiB
    if ab == FP64:
        m, n, k = 1024, 768, 768     # 6 + 4.5 + 6 MiB
    with installed() as fake, session(budget=16 * MiB) as s:
        _, info = run(s, ab, ct, 0, 1, m, n, k, 1.0, beta, 9)
        assert info.tile_count > 1 and info.maximum_working_set_bytes <= 16 * MiB
        tel = s.telemetry()
        assert tel.handle_reuses > 0
        assert tel.resident_bytes_peak <= 16 * MiB
        del fake


def test_auto_mode_follows_the_reference_mapping():
    """AUTO: TF32 on FP32 data (here the FP32-accurate three-term kernel), strict FP32 on
    FP16 / BF16, FP64 on FP64; explicit modes as requested."""
    with installed(), session() as s:
        for ab, ct, mode, want in [
                (FP32, FP32, sdk.COMPUTE_AUTO, sdk.COMPUTE_FP32_TF32),
                (FP32, FP32, sdk.COMPUTE_FP32_STRICT, sdk.COMPUTE_FP32_STRICT),
                (FP16, FP32, sdk.COMPUTE_AUTO, sdk.COMPUTE_FP32_STRICT),
                (BF16, BF16, sdk.COMPUTE_AUTO, sdk.COMPUTE_FP32_STRICT),
                (FP64, FP64, sdk.COMPUTE_AUTO, sdk.COMPUTE_FP64),
                (FP64, FP64, sdk.COMPUTE_FP64, sdk.COMPUTE_FP64)]:
            A, B, C_ = (s.alloc(64 * 64 * 8) for _ in range(3))
            desc = s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=ab),
                               sdk.matrix(B, 64, 64, 64, data_type=ab),
                               sdk.matrix(C_, 64, 64, 64, data_type=ct), mode=mode)
            plan = s.plan(desc)
            assert s.plan_info(plan).effective_compute_mode == want, (ab, ct, mode)
            s.t.gemm_plan_release(plan)


def test_unsupported_type_combinations_are_invalid_arguments():
    """The reference's type rule: the plan is refused with INVALID_ARGUMENT
    (unsupported_type_combination), not UNSUPPORTED."""
    with installed(), session() as s:
        A, B, C_ = (s.alloc(64 * 64 * 8) for _ in range(3))
        bad = [
            (FP16, FP32, FP32, sdk.COMPUTE_AUTO),         # A and B differ
            (FP16, FP16, FP64, sdk.COMPUTE_AUTO),         # half inputs, FP64 C
            (FP16, FP16, BF16, sdk.COMPUTE_AUTO),         # half inputs, the other half C
            (FP16, FP16, FP16, sdk.COMPUTE_FP32_TF32),    # TF32 on half inputs
            (FP32, FP32, FP32, sdk.COMPUTE_FP64),         # FP64 arithmetic on FP32
            (FP64, FP64, FP64, sdk.COMPUTE_FP32_STRICT),  # FP32 arithmetic on FP64
            (FP64, FP64, FP32, sdk.COMPUTE_AUTO),         # FP64 inputs, FP32 C
        ]
        for ta, tb, tc, mode in bad:
            desc = s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=ta),
                               sdk.matrix(B, 64, 64, 64, data_type=tb),
                               sdk.matrix(C_, 64, 64, 64, data_type=tc), mode=mode)
            st, _ = s.try_plan(desc)
            assert st == sdk.INVALID_ARGUMENT, (ta, tb, tc, mode)


def test_misaligned_offsets_are_refused_before_any_device_work():
    with installed(), session() as s:
        A, B, C_ = (s.alloc(64 * 64 * 8 + 64) for _ in range(3))
        desc = s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=FP64, offset=4),
                           sdk.matrix(B, 64, 64, 64, data_type=FP64),
                           sdk.matrix(C_, 64, 64, 64, data_type=FP64))
        st, _ = s.try_plan(desc)
        assert st == sdk.INVALID_ARGUMENT
        ok = s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=FP16, offset=2),
                         sdk.matrix(B, 64, 64, 64, data_type=FP16),
                         sdk.matrix(C_, 64, 64, 64, data_type=FP16))
        st, plan = s.try_plan(ok)
        assert st == sdk.SUCCESS
        s.t.gemm_plan_release(plan)


def test_element_sizes_bound_the_storage_checks():
    """An FP64 matrix needs twice the bytes of an FP32 one of the same shape."""
    with installed(), session() as s:
        A = s.alloc(64 * 64 * 4)
        B, C_ = s.alloc(64 * 64 * 8), s.alloc(64 * 64 * 8)
        for ab, want in ((FP32, sdk.SUCCESS), (FP64, sdk.INVALID_ARGUMENT)):
            desc = s.gemm_desc(sdk.matrix(A, 64, 64, 64, data_type=ab),
                               sdk.matrix(B, 64, 64, 64, data_type=ab),
                               sdk.matrix(C_, 64, 64, 64, data_type=ab))
            st, plan = s.try_plan(desc)
            assert st == want, ab
            if st == sdk.SUCCESS:
                s.t.gemm_plan_release(plan)
        assert ESIZE[FP64] == 2 * ESIZE[FP32]
