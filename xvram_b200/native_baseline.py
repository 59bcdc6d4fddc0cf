"""The ordinary cuBLAS SGEMM the reference makes, for comparison only.

The reference's strict-FP32 contraction is a cuBLAS call with CUBLAS_COMPUTE_32F_PEDANTIC
(src/gemm/executor.cpp:211-218; the core path src/platform/cublas/cublas_api.cpp:634-686:
cublasSetStream, cublasSetMathMode, cublasGemmEx with CUBLAS_GEMM_DEFAULT), and its compat
bench runs the same call as its "native baseline" (src/compat_bench/native_baseline.cpp:
70-90, math mode CUBLAS_PEDANTIC_MATH).  This module makes that call through ctypes on
device pointers, so bench.py can time the reference's own library contraction on this
GPU beside this library's kernel, and the compat bench can fill its native_baseline_*
fields.  Nothing in this library's product path calls it.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

CUDA_R_32F = 0
CUBLAS_COMPUTE_32F_PEDANTIC = 69
CUBLAS_PEDANTIC_MATH = 2
CUBLAS_GEMM_DEFAULT = -1


def _load() -> C.CDLL:
    names = []
    try:
        import nvidia.cublas
        names.append(str(Path(nvidia.cublas.__path__[0]) / "lib" / "libcublas.so.12"))
    except (ImportError, IndexError, AttributeError):
        pass
    names += ["libcublas.so.12", "/usr/local/cuda/lib64/libcublas.so.12"]
    last = None
    for name in names:
        if name.startswith("/") and not os.path.exists(name):
            continue
        try:
            return C.CDLL(name)
        except OSError as e:
            last = e
    raise RuntimeError(f"cuBLAS is not available: {last}")


class PedanticSgemm:
    """One cuBLAS handle bound to a stream, in pedantic math mode."""

    def __init__(self, stream_ptr: int = 0):
        self._lib = lib = _load()
        lib.cublasCreate_v2.argtypes = [C.POINTER(C.c_void_p)]
        lib.cublasSetStream_v2.argtypes = [C.c_void_p, C.c_void_p]
        lib.cublasSetMathMode.argtypes = [C.c_void_p, C.c_int]
        lib.cublasDestroy_v2.argtypes = [C.c_void_p]
        lib.cublasGemmEx.argtypes = [
            C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
            C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
            C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
        for f in (lib.cublasCreate_v2, lib.cublasSetStream_v2, lib.cublasSetMathMode,
                  lib.cublasDestroy_v2, lib.cublasGemmEx):
            f.restype = C.c_int
        self._h = C.c_void_p()
        self._check(lib.cublasCreate_v2(C.byref(self._h)), "cublasCreate_v2")
        self._check(lib.cublasSetStream_v2(self._h, C.c_void_p(stream_ptr)), "cublasSetStream_v2")
        self._check(lib.cublasSetMathMode(self._h, CUBLAS_PEDANTIC_MATH), "cublasSetMathMode")

    @staticmethod
    def _check(status: int, what: str) -> None:
        if status != 0:
            raise RuntimeError(f"{what} failed with cuBLAS status {status}")

    def __call__(self, op_a: int, op_b: int, m: int, n: int, k: int, alpha: float, a: int,
                 lda: int, b: int, ldb: int, beta: float, c: int, ldc: int) -> None:
        al, be = C.c_float(alpha), C.c_float(beta)
        self._check(self._lib.cublasGemmEx(
            self._h, op_a, op_b, m, n, k, C.byref(al), C.c_void_p(a), CUDA_R_32F, lda,
            C.c_void_p(b), CUDA_R_32F, ldb, C.byref(be), C.c_void_p(c), CUDA_R_32F, ldc,
            CUBLAS_COMPUTE_32F_PEDANTIC, CUBLAS_GEMM_DEFAULT), "cublasGemmEx")

    def version(self) -> int:
        """cublasGetVersion_v2: major * 10000 + minor * 100 + patch (12.9.1 -> 120901)."""
        v = C.c_int(0)
        self._lib.cublasGetVersion_v2.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        self._lib.cublasGetVersion_v2.restype = C.c_int
        self._check(self._lib.cublasGetVersion_v2(self._h, C.byref(v)), "cublasGetVersion_v2")
        return int(v.value)

    def close(self) -> None:
        if self._h:
            self._lib.cublasDestroy_v2(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
