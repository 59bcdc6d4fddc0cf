"""Parity of the sm_100a SGEMM kernels with the CPU FP64 oracle (device entry point).

Tolerance: max|err| / (K * max|a| * max|b|) <= 1e-6 (TOLERANCE), plus the reference's
own acceptance test |err| <= 1e-4 + 2e-5 |ref| where it applies."""
from __future__ import annotations

import numpy as np
import pytest

from oracle_lib import TOLERANCE, normalized_error, reference_criterion

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import device  # noqa: E402

AUTO, TMA, GENERIC = device.PATH_AUTO, device.PATH_TMA, device.PATH_GENERIC


def operands(oracle, op_a, op_b, m, n, k, pad, seed):
    ra, ca = (k, m) if op_a else (m, k)
    rb, cb = (n, k) if op_b else (k, n)
    lda, ldb, ldc = ra + pad[0], rb + pad[1], m + pad[2]
    a = oracle.uniform(ca * lda, seed).reshape(ca, lda)
    b = oracle.uniform(cb * ldb, seed + 1).reshape(cb, ldb)
    c = oracle.uniform(n * ldc, seed + 2).reshape(n, ldc)
    return a, lda, b, ldb, c, ldc


def run(oracle, op_a, op_b, m, n, k, alpha, beta, pad=(0, 0, 0), seed=0, path=AUTO,
        c_override=None):
    a, lda, b, ldb, c, ldc = operands(oracle, op_a, op_b, m, n, k, pad, seed)
    if c_override is not None:
        c = c_override(c)
    A, B, Cd = (torch.from_numpy(x).cuda() for x in (a, b, c))
    st = device.sgemm(op_a, op_b, m, n, k, alpha, A, lda, B, ldb, beta, Cd, ldc, path=path)
    assert st == 0
    assert device.kernel_status() == 0
    out = Cd.cpu().numpy()
    cin = None if beta == 0 else c
    ref = oracle.gemm(op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, cin, ldc)
    return out, ref, c, a, b


def check(out, ref, c, m, k, a, b):
    amax = float(np.abs(a).max()) if a.size else 1.0
    bmax = float(np.abs(b).max()) if b.size else 1.0
    err = normalized_error(out[:, :m], ref, max(k, 1), amax, bmax)
    assert err <= TOLERANCE, err
    assert np.array_equal(out[:, m:], c[:, m:])  # padding rows of C untouched
    return err


OPS = [(0, 0), (0, 1), (1, 0), (1, 1)]
SHAPES = [(1, 1, 1), (127, 129, 33), (129, 255, 257), (300, 200, 1000), (1000, 3, 64),
          (5, 1000, 64), (256, 256, 32), (513, 385, 129)]


@pytest.mark.parametrize("op_a,op_b", OPS)
@pytest.mark.parametrize("shape", SHAPES)
def test_tma_kernel_ragged_shapes(oracle, op_a, op_b, shape):
    m, n, k = shape
    ra = k if op_a else m
    rb = n if op_b else k
    pad = ((-ra) % 4 + 4, (-rb) % 4, 3)  # TMA needs ld % 4 == 0
    out, ref, c, a, b = run(oracle, op_a, op_b, m, n, k, 0.5, 1.5, pad=pad, path=TMA)
    check(out, ref, c, m, k, a, b)


@pytest.mark.parametrize("op_a,op_b", OPS)
@pytest.mark.parametrize("shape", SHAPES[:5])
def test_generic_kernel_any_alignment(oracle, op_a, op_b, shape):
    m, n, k = shape
    out, ref, c, a, b = run(oracle, op_a, op_b, m, n, k, -2.0, 0.25, pad=(1, 3, 5), path=GENERIC)
    check(out, ref, c, m, k, a, b)


def test_auto_falls_back_for_unaligned_ld(oracle):
    out, ref, c, a, b = run(oracle, 0, 0, 37, 19, 67, 1.0, 0.0, pad=(0, 0, 0), path=AUTO)
    check(out, ref, c, 37, 67, a, b)
    st = device.sgemm(0, 0, 37, 19, 67, 1.0, torch.zeros(67 * 37, device="cuda"), 37,
                      torch.zeros(19 * 67, device="cuda"), 67, 0.0,
                      torch.zeros(19 * 37, device="cuda"), 37, path=TMA)
    assert st == 1  # INVALID_ARGUMENT: TMA cannot take ld = 37


def test_preview_gemm_pattern(oracle):
    """examples/preview-gemm operands, 37x19x67 NN, reference acceptance criterion."""
    m, n, k = 37, 19, 67
    a = np.array([[oracle.lib.xo_pv_a(r, c) for r in range(m)] for c in range(k)], np.float32)
    b = np.array([[oracle.lib.xo_pv_b(r, c) for r in range(k)] for c in range(n)], np.float32)
    for path, ld_pad in ((GENERIC, 0), (TMA, 3)):
        ap = np.zeros((k, m + ld_pad), np.float32); ap[:, :m] = a
        bp = np.zeros((n, k + (1 if ld_pad else 0)), np.float32); bp[:, :k] = b
        if path == TMA:
            bp = np.zeros((n, 68), np.float32); bp[:, :k] = b
        A, B = torch.from_numpy(ap).cuda(), torch.from_numpy(bp).cuda()
        Cd = torch.full((n, m), float("nan"), device="cuda")
        assert device.sgemm(0, 0, m, n, k, 1.0, A, ap.shape[1], B, bp.shape[1], 0.0, Cd, m,
                            path=path) == 0
        out = Cd.cpu().numpy()
        ref = oracle.gemm(0, 0, m, n, k, 1.0, ap, ap.shape[1], bp, bp.shape[1], 0.0, None, m)
        assert reference_criterion(out, ref)
        assert np.array_equal(out.astype(np.float64), ref)  # small integers/16: exact


@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.0, 1.0), (0.0, 0.0), (1.0, 1.0), (-0.75, -2.0)])
def test_alpha_beta_cases(oracle, alpha, beta):
    out, ref, c, a, b = run(oracle, 1, 0, 300, 260, 96, alpha, beta, pad=(0, 0, 4), path=TMA)
    check(out, ref, c, 300, 96, a, b)


@pytest.mark.parametrize("path", [TMA, GENERIC])
def test_beta_zero_does_not_read_c(oracle, path):
    out, ref, c, a, b = run(oracle, 0, 1, 200, 130, 64, 1.0, 0.0, pad=(0, 2, 0), path=path,
                            c_override=lambda c: np.full_like(c, np.nan))
    assert np.all(np.isfinite(out))
    check(out, ref, c, 200, 64, a, b)


def test_k_zero_scales_c(oracle):
    c = oracle.uniform(40 * 30, 5).reshape(30, 40)
    Cd = torch.from_numpy(c).cuda()
    dummy = torch.zeros(4, device="cuda")
    assert device.sgemm(0, 0, 40, 30, 0, 1.0, dummy, 40, dummy, 1, 2.0, Cd, 40) == 0
    assert np.array_equal(Cd.cpu().numpy(), (2.0 * c).astype(np.float32))


def test_c1_1024_cubed_full_check(oracle):
    """1024^3 NN, alpha 1, beta 0, seeds 0/1, C zero; full FP64 check."""
    n = 1024
    a = oracle.uniform(n * n, 0).reshape(n, n)
    b = oracle.uniform(n * n, 1).reshape(n, n)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    Cd = torch.zeros((n, n), device="cuda")
    assert device.sgemm(0, 0, n, n, n, 1.0, A, n, B, n, 0.0, Cd, n) == 0
    assert device.kernel_status() == 0
    out = Cd.cpu().numpy()
    ref = oracle.gemm(0, 0, n, n, n, 1.0, a, n, b, n, 0.0, None, n, threads=16)
    err = normalized_error(out, ref, n, float(np.abs(a).max()), float(np.abs(b).max()))
    assert err <= TOLERANCE
    assert reference_criterion(out, ref)


def test_c2_full_size_sampled_and_checksum(oracle):
    """M=8192 N=6144 K=4096 TN, alpha 0.5, beta 1.5 (A stored K x M).
    65536 sampled outputs against FP64, plus the size-independent identity
    sum_ij C_ij = alpha * sum_p rowsum(op(A))_p colsum(op(B))_p + beta * sum C_in."""
    m, n, k = 8192, 6144, 4096
    a = oracle.uniform(k * m, 10).reshape(m, k)      # stored K x M column-major
    b = oracle.uniform(k * n, 11).reshape(n, k)      # stored K x N column-major
    c = oracle.uniform(m * n, 12).reshape(n, m)
    A, B, Cd = (torch.from_numpy(x).cuda() for x in (a, b, c))
    assert device.sgemm(1, 0, m, n, k, 0.5, A, k, B, k, 1.5, Cd, m) == 0
    assert device.kernel_status() == 0
    out = Cd.cpu().numpy()
    rng = np.random.default_rng(0)
    rows, cols = rng.integers(0, m, 65536), rng.integers(0, n, 65536)
    ref = oracle.gemm_sampled(1, 0, k, 0.5, a, k, b, k, 1.5, c, m, rows, cols, threads=16)
    err = float(np.max(np.abs(out[cols, rows].astype(np.float64) - ref))) / k
    assert err <= TOLERANCE
    lhs = out.astype(np.float64).sum()
    sa = a.astype(np.float64).sum(axis=0)   # sum_i op(A)(i, p), p = 0..k-1
    sb = b.astype(np.float64).sum(axis=0)   # sum_j op(B)(p, j)
    rhs = 0.5 * float(sa @ sb) + 1.5 * c.astype(np.float64).sum()
    assert abs(lhs - rhs) <= TOLERANCE * k * (m * n) ** 0.5  # per-element bound x sqrt(count)


def test_repeat_calls_are_deterministic(oracle):
    m, n, k = 1000, 900, 800
    a = oracle.uniform(m * k, 21).reshape(k, m)
    b = oracle.uniform(k * n, 22).reshape(n, k)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    outs = []
    for _ in range(3):
        Cd = torch.zeros((n, m), device="cuda")
        assert device.sgemm(0, 0, m, n, k, 1.0, A, m, B, k, 0.0, Cd, m) == 0
        outs.append(Cd.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


@pytest.mark.parametrize("packed", [False, True])
def test_ffma_probe_runs(packed):
    sink = torch.zeros(1, device="cuda")
    assert device.ffma_probe(148, 8, sink, packed=packed) == 0
    torch.cuda.synchronize()
    assert float(sink[0]) == 0.0


@pytest.mark.parametrize("op_a,op_b", [(1, 0), (0, 0), (1, 1)])
def test_canonicalised_path_is_bit_identical(oracle, op_a, op_b):
    """K-major operands transposed into scratch + the M/N-major kernel give exactly the
    bits of the direct K-major kernel (same FFMA order per output)."""
    m, n, k = 700, 520, 300
    a, lda, b, ldb, c, ldc = operands(oracle, op_a, op_b, m, n, k, (0, 0, 0), 50)
    lda_p = lda + (-lda) % 4
    ldb_p = ldb + (-ldb) % 4
    ap = np.zeros((a.shape[0], lda_p), np.float32); ap[:, :lda] = a
    bp = np.zeros((b.shape[0], ldb_p), np.float32); bp[:, :ldb] = b
    A, B = torch.from_numpy(ap).cuda(), torch.from_numpy(bp).cuda()
    need = device.workspace_bytes(op_a, op_b, m, n, k)
    assert need > 0
    ws = torch.empty(need // 4 + 64, device="cuda")
    outs = []
    for mode in ("pool", "explicit", "direct"):
        Cd = torch.from_numpy(c).cuda()
        if mode == "pool":
            st = device.sgemm(op_a, op_b, m, n, k, 0.5, A, lda_p, B, ldb_p, 1.5, Cd, ldc)
        elif mode == "explicit":
            st = device.sgemm_ws(op_a, op_b, m, n, k, 0.5, A, lda_p, B, ldb_p, 1.5, Cd, ldc, ws,
                                 need)
        else:  # too little workspace: the K-major kernel runs directly
            st = device.sgemm_ws(op_a, op_b, m, n, k, 0.5, A, lda_p, B, ldb_p, 1.5, Cd, ldc, ws, 0)
        assert st == 0
        assert device.kernel_status() == 0
        outs.append(Cd.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    ref = oracle.gemm(op_a, op_b, m, n, k, 0.5, ap, lda_p, bp, ldb_p, 1.5, c, ldc)
    check(outs[0], ref, c, m, k, a, b)


def test_workspace_query():
    assert device.workspace_bytes(0, 1, 100, 100, 100) == 0
    assert device.workspace_bytes(1, 1, 100, 100, 100) == 100 * 100 * 4 + (256 - 100 * 100 * 4 % 256) % 256
    assert device.workspace_bytes(1, 0, 101, 99, 7) >= (104 * 7 + 100 * 7) * 4


@pytest.mark.parametrize("op_a,op_b", [(0, 1), (1, 0)])
@pytest.mark.parametrize("shape,tile", [
    ((2560, 2048, 96), (128, 256)),    # 160 tiles: 12-tile tail, split
    ((1300, 700, 64), (128, 256)),     # 33 tiles: all half-width
    ((2560, 1280, 64), (128, 256)),    # 100 tiles: tail too big to split
    ((2000, 3000, 700), (128, 256)),   # 192 tiles: 44-tile tail, split
    ((2560, 1280, 256), (128, 256)),   # 100 tiles: one partial wave
    ((4096, 8192, 160), (192, 192)),   # 946 tiles: 58-tile tail, split
    ((2688, 2688, 96), (192, 192)),    # 196 tiles: 48-tile tail, split
    ((4224, 2304, 64), (192, 192)),    # 264 tiles: 116-tile tail, not split
    ((2300, 2292, 100), (192, 192)),   # 144 ragged tiles, one partial wave, ragged k
    ((8192, 6144, 64), (192, 192))])   # C2's M and N: 1376 tiles, 44-tile tail, split
def test_tail_split_is_bit_identical_to_generic(oracle, op_a, op_b, shape, tile):
    """Both tilings of the TMA kernel (12 warps on 192 x 192 tiles, 8 warps on 128 x 256)
    run a last, at most half-full wave as half-width tiles; every output is still one FFMA
    chain in k order, so its bits equal the generic kernel's.  The tiling each shape gets
    (on a 148-SM B200) is checked first, so both forms and both tail cases are covered."""
    m, n, k = shape
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert device.tile_shape(m, n) == tile
    outs = []
    for path in (TMA, GENERIC):
        out, ref, c, a, b = run(oracle, op_a, op_b, m, n, k, 0.5, 1.5, seed=70, path=path)
        outs.append(out)
    assert np.array_equal(outs[0], outs[1])
    check(outs[0], ref, c, m, k, a, b)



@pytest.mark.parametrize("op_a,op_b", OPS)
@pytest.mark.parametrize("shape", [(513, 385, 129), (1024, 768, 1000), (300, 200, 4096)])
def test_matches_the_reference_library_contraction(oracle, op_a, op_b, shape):
    """Against the reference's own GPU contraction on the same device inputs: cuBLAS
    cublasGemmEx with CUBLAS_COMPUTE_32F_PEDANTIC in pedantic math mode
    (xvram_b200.native_baseline; reference src/gemm/executor.cpp:211-218).  Both are strict
    FP32 with different summation orders, so they agree within the SGEMM tolerance of each
    other, and each is within it of the FP64 oracle."""
    from xvram_b200.native_baseline import PedanticSgemm
    m, n, k = shape
    a, lda, b, ldb, c, ldc = operands(oracle, op_a, op_b, m, n, k, (0, 0, 0), 70)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    ours, lib = torch.from_numpy(c).cuda(), torch.from_numpy(c).cuda()
    assert device.sgemm(op_a, op_b, m, n, k, 0.5, A, lda, B, ldb, 1.5, ours, ldc) == 0
    assert device.kernel_status() == 0
    try:
        gemm = PedanticSgemm(torch.cuda.current_stream().cuda_stream)
    except RuntimeError as e:
        pytest.skip(str(e))
    with gemm:
        gemm(op_a, op_b, m, n, k, 0.5, A.data_ptr(), lda, B.data_ptr(), ldb, 1.5,
             lib.data_ptr(), ldc)
    torch.cuda.synchronize()
    o, l = ours.cpu().numpy(), lib.cpu().numpy()
    ref = oracle.gemm(op_a, op_b, m, n, k, 0.5, a, lda, b, ldb, 1.5, c, ldc)
    amax, bmax = float(np.abs(a).max()), float(np.abs(b).max())
    assert normalized_error(o[:, :m], l[:, :m].astype(np.float64), k, amax, bmax) <= TOLERANCE
    assert normalized_error(o[:, :m], ref, k, amax, bmax) <= TOLERANCE
    assert normalized_error(l[:, :m], ref, k, amax, bmax) <= TOLERANCE
