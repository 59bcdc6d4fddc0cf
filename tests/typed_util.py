"""Test data and checks for the FP16 / BF16 / FP64 GEMMs (the reference's other element
types, src/gemm/planner.cpp:819-842).

Inputs are seeded uniform[-1, 1) values (the oracle's generator) rounded to the element
type; the FP16 / BF16 reference is the oracle's FP64 GEMM of the exactly widened values,
the FP64 reference the oracle's long-double GEMM.  Tolerances, per output element:
  * FP32 C from FP16 / BF16 inputs: the FP32 bound, max|err| / (K max|a| max|b|) <= 1e-6;
  * FP16 / BF16 C: that bound plus one rounding to the type, 2^-11 (FP16) or 2^-8 (BF16)
    of |ref|;
  * FP64: max|err| / (K max|a| max|b|) <= 1e-13 (the kernel's FP64 arithmetic gives about
    1e-16; FP32 arithmetic would give about 1e-8).
"""
from __future__ import annotations

import numpy as np

from oracle_lib import TOLERANCE, load_oracle

FP16, BF16, FP32, FP64 = range(4)
ESIZE = {FP16: 2, BF16: 2, FP32: 4, FP64: 8}
FP64_TOLERANCE = 1e-13


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def from_bf16_bits(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def encode(values: np.ndarray, dtype: int) -> np.ndarray:
    """float32/64 values -> the stored array of `dtype` (FP16/BF16 as uint16 bits)."""
    if dtype == FP16:
        return values.astype(np.float16).view(np.uint16)
    if dtype == BF16:
        return to_bf16_bits(values.astype(np.float32))
    if dtype == FP32:
        return values.astype(np.float32)
    return values.astype(np.float64)


def decode(stored: np.ndarray, dtype: int) -> np.ndarray:
    """Stored array -> exact float64 values."""
    if dtype == FP16:
        return stored.view(np.float16).astype(np.float64)
    if dtype == BF16:
        return from_bf16_bits(stored).astype(np.float64)
    return stored.astype(np.float64)


def make_problem(ab: int, ct: int, op_a: int, op_b: int, m: int, n: int, k: int, seed: int):
    """Stored A, B, C (column-major, tight leading dimensions) and their exact values."""
    orc = load_oracle()
    if ab == FP64:
        # FP64 data with full 53-bit significands: the sum of two float32 draws at
        # different scales.
        a = orc.uniform(m * k, seed).astype(np.float64) + \
            orc.uniform(m * k, seed + 10).astype(np.float64) * 2.0 ** -30
        b = orc.uniform(k * n, seed + 1).astype(np.float64) + \
            orc.uniform(k * n, seed + 11).astype(np.float64) * 2.0 ** -30
        c = orc.uniform(m * n, seed + 2).astype(np.float64)
    else:
        a = orc.uniform(m * k, seed)
        b = orc.uniform(k * n, seed + 1)
        c = orc.uniform(m * n, seed + 2)
    A, B, Cs = encode(a, ab), encode(b, ab), encode(c, ct)
    return A, B, Cs, decode(A, ab), decode(B, ab), decode(Cs, ct)


def reference(ab, op_a, op_b, m, n, k, alpha, av, bv, beta, cv):
    """(n, m) float64 reference of alpha op(A) op(B) + beta C from exact input values."""
    orc = load_oracle()
    lda, ldb = (m if op_a == 0 else k), (k if op_b == 0 else n)
    if ab == FP64:
        return orc.gemm_f64_inputs(op_a, op_b, m, n, k, alpha, av, lda, bv, ldb, beta,
                                   cv if beta != 0 else None, m)
    return orc.gemm(op_a, op_b, m, n, k, alpha, av.astype(np.float32), lda,
                    bv.astype(np.float32), ldb, beta,
                    cv.astype(np.float32) if beta != 0 else None, m)


def check(ab, ct, out_stored, ref, k, amax=1.0, bmax=1.0) -> float:
    """Asserts the per-element bound of the module docstring; returns the normalised
    error against the reference."""
    out = decode(out_stored, ct).reshape(ref.shape)
    err = np.abs(out - ref)
    scale = k * amax * bmax
    if ab == FP64:
        bound = FP64_TOLERANCE * scale
    else:
        bound = TOLERANCE * scale + (2.0 ** -11 if ct == FP16 else 2.0 ** -8 if ct == BF16
                                     else 0.0) * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (int(bad.sum()), float(err.max()), float(np.max(bound)))
    return float(err.max() / scale)
