"""ctypes bindings of the CPU oracle (oracle/) for the tests and the benchmark's CPU legs.

Test infrastructure: the oracle is the checker and the CPU baseline, never the path
being measured.  `load_oracle()` builds oracle/_build/libxvram_oracle.so with make if
it is missing; `load_reference()` returns the reference-compiled oracle/_ref library
or None when it has not been built.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_SO = ROOT / "oracle" / "_build" / "libxvram_oracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "libxvram_ref.so"

u32, u64, i32, i64, f32, f64, vp = (C.c_uint32, C.c_uint64, C.c_int32, C.c_int64, C.c_float,
                                    C.c_double, C.c_void_p)


class Oracle:
    def __init__(self, lib: C.CDLL):
        self.lib = lib
        lib.xo_uniform_at.argtypes = [u64, u64]
        lib.xo_uniform_at.restype = f32
        lib.xo_fill_uniform.argtypes = [vp, u64, u64, u64]
        lib.xo_fill_uniform.restype = None
        lib.xo_gemm_f64.argtypes = [C.c_int, C.c_int, i64, i64, i64, f64, vp, i64, vp, i64, f64,
                                    vp, i64, vp, i64, C.c_int]
        lib.xo_gemm_f64.restype = C.c_int
        lib.xo_gemm_f64_sampled.argtypes = [C.c_int, C.c_int, i64, f64, vp, i64, vp, i64, f64, vp,
                                            i64, vp, vp, i64, vp, C.c_int]
        lib.xo_gemm_f64_sampled.restype = C.c_int
        for name in ("xo_cb_pattern_a", "xo_cb_pattern_b"):
            getattr(lib, name).argtypes = [u64, u64, u64]
            getattr(lib, name).restype = f32
        lib.xo_cb_pattern_c.argtypes = [u64, u64]
        lib.xo_cb_pattern_c.restype = f32
        lib.xo_cb_reference_dot.argtypes = [u64, u64, u64, u64, C.c_int]
        lib.xo_cb_reference_dot.restype = f64
        lib.xo_cb_reference_result.argtypes = [u64, u64, u64, u64, f32, f32, u32, C.c_int]
        lib.xo_cb_reference_result.restype = f64
        lib.xo_gb_a.argtypes = [u64, u64]
        lib.xo_gb_a.restype = u64
        lib.xo_gb_b.argtypes = [u64, u64]
        lib.xo_gb_b.restype = u64
        lib.xo_gb_expected.argtypes = [u64, u64, u64]
        lib.xo_gb_expected.restype = u64
        lib.xo_pv_a.argtypes = [C.c_int, C.c_int]
        lib.xo_pv_a.restype = f32
        lib.xo_pv_b.argtypes = [C.c_int, C.c_int]
        lib.xo_pv_b.restype = f32
        lib.xo_gemm_f64_inputs.argtypes = [C.c_int, C.c_int, i64, i64, i64, f64, vp, i64, vp,
                                           i64, f64, vp, i64, vp, i64]
        lib.xo_gemm_f64_inputs.restype = C.c_int
        lib.xo_close_enough.argtypes = [f64, f64]
        lib.xo_close_enough.restype = C.c_int

    def uniform(self, count: int, seed: int, first: int = 0) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        self.lib.xo_fill_uniform(out.ctypes.data, count, seed, first)
        return out

    def gemm(self, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, threads=8):
        """FP64 reference result (m x n column-major, returned as an (n, m) array)."""
        out = np.empty((n, m), dtype=np.float64)
        cptr = c.ctypes.data if c is not None else None
        rc = self.lib.xo_gemm_f64(op_a, op_b, m, n, k, alpha, a.ctypes.data, lda, b.ctypes.data,
                                  ldb, beta, cptr, ldc, out.ctypes.data, m, threads)
        assert rc == 0
        return out

    def gemm_f64_inputs(self, op_a, op_b, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc):
        """FP64-input reference (long double accumulation), (n, m) array."""
        out = np.empty((n, m), dtype=np.float64)
        a = np.ascontiguousarray(a, dtype=np.float64)
        b = np.ascontiguousarray(b, dtype=np.float64)
        keep = c if c is None else np.ascontiguousarray(c, dtype=np.float64)
        cptr = keep.ctypes.data if keep is not None else None
        rc = self.lib.xo_gemm_f64_inputs(op_a, op_b, m, n, k, alpha, a.ctypes.data, lda,
                                         b.ctypes.data, ldb, beta, cptr, ldc, out.ctypes.data, m)
        assert rc == 0
        return out

    def gemm_sampled(self, op_a, op_b, k, alpha, a, lda, b, ldb, beta, c, ldc, rows, cols,
                     threads=8):
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        cols = np.ascontiguousarray(cols, dtype=np.int64)
        out = np.empty(rows.size, dtype=np.float64)
        cptr = c.ctypes.data if c is not None else None
        rc = self.lib.xo_gemm_f64_sampled(op_a, op_b, k, alpha, a.ctypes.data, lda, b.ctypes.data,
                                          ldb, beta, cptr, ldc, rows.ctypes.data,
                                          cols.ctypes.data, rows.size, out.ctypes.data, threads)
        assert rc == 0
        return out


def load_oracle() -> Oracle:
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "all"], check=True,
                       capture_output=True)
    return Oracle(C.CDLL(str(ORACLE_SO)))


def load_reference():
    if not REF_SO.exists():
        return None
    lib = C.CDLL(str(REF_SO))
    lib.xr_cb_pattern_a.argtypes = [u64, u64, u64]
    lib.xr_cb_pattern_a.restype = f32
    lib.xr_cb_pattern_b.argtypes = [u64, u64, u64]
    lib.xr_cb_pattern_b.restype = f32
    lib.xr_cb_pattern_c.argtypes = [u64, u64]
    lib.xr_cb_pattern_c.restype = f32
    lib.xr_cb_reference_dot.argtypes = [u64, u64, u64, u64, C.c_int]
    lib.xr_cb_reference_dot.restype = f64
    lib.xr_cb_reference_result.argtypes = [u64, u64, u64, u64, u64, u64, f32, f32, u32, C.c_int]
    lib.xr_cb_reference_result.restype = f64
    lib.xr_gb_expected.argtypes = [u64, u64, u64, C.POINTER(u64)]
    lib.xr_gb_expected.restype = C.c_int
    arr = C.POINTER(u64)
    lib.xr_validate_problem.argtypes = [u64, u64, u64, C.c_int, C.c_int, arr, arr, arr, arr, arr,
                                        arr, C.c_char_p]
    lib.xr_validate_problem.restype = C.c_int
    lib.xr_cpu_gemm_sample.argtypes = [u64, u64, u64, u64, u64, f32, f32, u64, C.c_int]
    lib.xr_cpu_gemm_sample.restype = f64
    return lib


def normalized_error(out: np.ndarray, ref: np.ndarray, k: int, amax: float, bmax: float) -> float:
    """max|out - ref| / (K * max|a| * max|b|): the tolerance metric of the SGEMM path."""
    denom = k * max(amax, 1e-30) * max(bmax, 1e-30)
    return float(np.max(np.abs(out.astype(np.float64) - ref)) / denom)


def reference_criterion(out: np.ndarray, ref: np.ndarray) -> bool:
    """The reference's acceptance test |err| <= 1e-4 + 2e-5 |ref|
    (src/compat_bench/executor.cpp:93-96)."""
    o = out.astype(np.float64)
    return bool(np.all(np.isfinite(o)) and np.all(np.abs(o - ref) <= 1e-4 + 2e-5 * np.abs(ref)))


TOLERANCE = 1e-6  # max|err| / (K max|a| max|b|), the bound stated for the SGEMM path
