"""The CPU oracle against the reference's own code (golden vectors + live _ref build)."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from oracle_lib import TOLERANCE, normalized_error, reference_criterion


def f32(h: str) -> float:
    return struct.unpack("<f", bytes.fromhex(h))[0]


def f64(h: str) -> float:
    return struct.unpack("<d", bytes.fromhex(h))[0]


def bits32(x: float) -> str:
    return struct.pack("<f", x).hex()


def test_compat_patterns_match_golden(oracle, golden):
    for seed, row, k, a, b, c in golden["cb_patterns"]:
        assert bits32(oracle.lib.xo_cb_pattern_a(row, k, seed)) == a
        assert bits32(oracle.lib.xo_cb_pattern_b(k, row, seed)) == b
        assert bits32(oracle.lib.xo_cb_pattern_c(row, k)) == c


def test_reference_dot_full_and_closed_form_match_golden(oracle, golden):
    for seed, row, col, k, full, closed in golden["cb_dots"]:
        assert oracle.lib.xo_cb_reference_dot(row, col, k, seed, 1) == f64(full)
        assert oracle.lib.xo_cb_reference_dot(row, col, k, seed, 0) == f64(closed)


def test_reference_result_matches_golden(oracle, golden):
    for seed, m, n, k, row, col, alpha, beta, passes, want in golden["cb_results"]:
        got = oracle.lib.xo_cb_reference_result(row, col, k, seed, alpha, beta, passes, 1)
        assert got == f64(want)


def test_gemm_bench_closed_form_matches_golden(oracle, golden):
    for row, col, k, a, b, expected in golden["gb_expected"]:
        assert oracle.lib.xo_gb_a(row, k) == a
        assert oracle.lib.xo_gb_b(k, col) == b
        assert expected is not None
        assert oracle.lib.xo_gb_expected(row, col, k) == expected
        if k <= 4096:  # the closed form is the exact sum
            s = sum(oracle.lib.xo_gb_a(row, p) * oracle.lib.xo_gb_b(p, col) for p in range(k))
            assert s == expected


def _padded(golden, ta, tb, operand):
    g = golden["cb_padded_fills"]
    for f in g["fills"]:
        if (f["ta"], f["tb"], f["operand"]) == (ta, tb, operand):
            return np.frombuffer(bytes.fromhex(f["bits"]), dtype=np.float32), f["ld"]
    raise KeyError


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_fp64_gemm_equals_reference_loop_on_padded_suite(oracle, golden, ta, tb):
    """xo_gemm_f64 over the reference's padded operands (37x19x67, padding 5, offset 11)
    is bit-identical to the reference's own FP64 reference_result."""
    shp = golden["cb_padded_fills"]["shape"]
    m, n, k, off = shp["m"], shp["n"], shp["k"], shp["offset"]
    a, lda = _padded(golden, ta, tb, 0)
    b, ldb = _padded(golden, ta, tb, 1)
    c, ldc = _padded(golden, ta, tb, 2)
    for alpha, beta in ((1.0, 0.0), (0.5, 1.5), (-2.0, 0.25)):
        out = oracle.gemm(ta, tb, m, n, k, alpha, a[off:], lda, b[off:], ldb, beta, c[off:], ldc)
        for j in range(n):
            for i in range(m):
                want = oracle.lib.xo_cb_reference_result(i, j, k, 0, alpha, beta, 1, 1)
                assert out[j, i] == want


def test_padded_fill_padding_value(golden):
    pad = f32(golden["cb_padded_fills"]["padding_value"])
    assert pad == -1234.5
    a, lda = _padded(golden, 0, 0, 0)
    assert np.all(a[:11] == pad)  # the leading offset is padding


def test_oracle_live_against_reference_build(oracle, ref_lib):
    for seed in (0, 1, 0x1234, 0x300):
        for row in range(7):
            for k in range(9):
                assert oracle.lib.xo_cb_pattern_a(row, k, seed) == ref_lib.xr_cb_pattern_a(row, k, seed)
                assert oracle.lib.xo_cb_pattern_b(k, row, seed) == ref_lib.xr_cb_pattern_b(k, row, seed)
        for k in (1, 7, 64, 1001):
            assert oracle.lib.xo_cb_reference_dot(3, 5, k, seed, 1) == ref_lib.xr_cb_reference_dot(3, 5, k, seed, 1)
            assert oracle.lib.xo_cb_reference_dot(3, 5, k, seed, 0) == ref_lib.xr_cb_reference_dot(3, 5, k, seed, 0)


def test_preview_gemm_known_answer(oracle):
    """examples/preview-gemm: 37x19x67 NN, alpha 1, beta 0, checked against FP64."""
    m, n, k = 37, 19, 67
    a = np.array([[oracle.lib.xo_pv_a(r, c) for r in range(m)] for c in range(k)], np.float32)
    b = np.array([[oracle.lib.xo_pv_b(r, c) for r in range(k)] for c in range(n)], np.float32)
    out = oracle.gemm(0, 0, m, n, k, 1.0, a, m, b, k, 0.0, None, m)
    ref = (b.astype(np.float64) @ a.astype(np.float64))  # (n, m) = (A B)^T
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_fp64_gemm_matches_numpy(oracle, ta, tb):
    rng = np.random.default_rng(7)
    m, n, k = 29, 23, 41
    lda = (k if ta else m) + 3
    ldb = (n if tb else k) + 2
    ldc = m + 1
    a = rng.uniform(-1, 1, size=((m if ta else k), lda)).astype(np.float32)
    b = rng.uniform(-1, 1, size=((k if tb else n), ldb)).astype(np.float32)
    c = rng.uniform(-1, 1, size=(n, ldc)).astype(np.float32)
    A = (a[:, :k].T if ta else a[:, :m].T)  # op(A) as m x k... build explicitly below
    opA = np.empty((m, k)); opB = np.empty((k, n))
    for i in range(m):
        for p in range(k):
            opA[i, p] = a[i, p] if ta else a[p, i]
    for p in range(k):
        for j in range(n):
            opB[p, j] = b[p, j] if tb else b[j, p]
    want = 0.5 * (opA @ opB) + 1.5 * c[:, :m].T.astype(np.float64)
    out = oracle.gemm(ta, tb, m, n, k, 0.5, a, lda, b, ldb, 1.5, c, ldc)
    assert np.allclose(out.T, want, rtol=0, atol=1e-12)
    del A


def test_sampled_equals_full(oracle):
    rng = np.random.default_rng(3)
    m, n, k = 50, 40, 70
    a = rng.uniform(-1, 1, (k, m)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    c = rng.uniform(-1, 1, (n, m)).astype(np.float32)
    full = oracle.gemm(0, 0, m, n, k, 1.25, a, m, b, k, -0.5, c, m)
    rows = rng.integers(0, m, 200)
    cols = rng.integers(0, n, 200)
    s = oracle.gemm_sampled(0, 0, k, 1.25, a, m, b, k, -0.5, c, m, rows, cols)
    assert np.array_equal(s, full[cols, rows])


def test_generator_range_and_exactness(oracle):
    x = oracle.uniform(1 << 16, seed=0)
    assert x.min() >= -1.0 and x.max() < 1.0
    assert np.all(x * 8388608.0 == np.round(x * 8388608.0))
    assert oracle.lib.xo_uniform_at(0, 12345) == x[12345]
    y = oracle.uniform(100, seed=0, first=12300)
    assert np.array_equal(y, x[12300:12400])
    assert not np.array_equal(oracle.uniform(100, seed=1), x[:100])


def test_tolerance_helpers():
    ref = np.array([1.0, -2.0, 3.0])
    out = np.array([1.0, -2.0, 3.0 + 5e-5], np.float32)
    assert reference_criterion(out, ref)
    assert normalized_error(out, ref, 4096, 1.0, 1.0) < TOLERANCE
    assert not reference_criterion(np.array([np.nan, 0, 0], np.float32), ref)
