"""The drop-in boundary, proved with the reference's own contracts and consumers.

Each test runs a contract script or builds a consumer program of the reference, read in
place from the reference tree, against this repository's headers (include/xvram/...) and
libraries.  None needs a GPU.  They skip where the reference tree is absent.

* cuda_compat_export_contract.py / sdk_export_contract.py (tests/contract): the compat
  library exports exactly xvram_cuda_compat_get_api@@XVRAM_CUDA_COMPAT_1.0 and the SDK
  library exactly xvram_get_api@@XVRAM_0.1.
* cuda_compat_consumer_contract.py with tests/compat_consumer: the C++ facade
  <xvram/cuda_compat.hpp> builds with -Wall -Wextra -Wpedantic -Werror, remaps the
  approved cudaMalloc / cublasSgemm spellings, runs without a driver, and leaves every
  other CUDA / cuBLAS call (cudaMemset, cuInit, cublasDgemm, cudaLaunchKernel) and device
  compilation failing at build time.
* tests/unit/cuda_compat_facade_tests.cpp: the facade refuses cleanly on a rejected
  negotiation, on a table with missing members and on a table of another version, keeps
  the last error per thread, and negotiates once.
* tests/package_consumer/cuda_compat.c and examples/preview-gemm/main.cpp: the reference's
  C and C++ consumers of <xvram/cuda_compat.h> build against this library and run as far
  as a machine without a GPU allows (tests/test_c_consumer_gpu.py runs the GEMM example on
  a B200).
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

import pytest

from reference_tree import reference_file

ROOT = Path(__file__).resolve().parents[1]
INCLUDE = ROOT / "include"
CUDA_INCLUDE = Path("/usr/local/cuda/include")


def _lib(name: str) -> Path:
    from xvram_b200 import _native
    return {"compat": _native.COMPAT_LIB_PATH, "sdk": _native.SDK_LIB_PATH}[name]


def _need(*parts: str) -> Path:
    p = reference_file(*parts)
    if p is None:
        pytest.skip("reference tree not present")
    return p


def _run(cmd, **kw) -> subprocess.CompletedProcess:
    return subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=300,
                          **kw)


@pytest.mark.parametrize("script,lib", [("cuda_compat_export_contract.py", "compat"),
                                        ("sdk_export_contract.py", "sdk")])
def test_reference_export_contract(script, lib):
    path = _need("tests", "contract", script)
    selftest = _run([sys.executable, path, "--self-test"], cwd=path.parent)
    assert selftest.returncode == 0, selftest.stdout + selftest.stderr
    r = _run([sys.executable, path, _lib(lib)], cwd=path.parent)
    assert r.returncode == 0, r.stdout + r.stderr


def test_reference_export_contract_rejects_the_native_library():
    """The native library (many exports) is not the drop-in, and the contract says so."""
    from xvram_b200 import _native
    path = _need("tests", "contract", "cuda_compat_export_contract.py")
    r = _run([sys.executable, path, _native.PRODUCT_LIB_PATH], cwd=path.parent)
    assert r.returncode != 0 and "expected exports" in r.stdout


@pytest.mark.skipif(shutil.which("cmake") is None or shutil.which("ninja") is None,
                    reason="needs cmake and ninja")
def test_reference_compat_consumer_profile(tmp_path):
    script = _need("tests", "contract", "cuda_compat_consumer_contract.py")
    source = _need("tests", "compat_consumer")
    lib = _lib("compat")
    r = _run([sys.executable, script, "--cmake", shutil.which("cmake"), "--source", source,
              "--library", lib, "--link-library", lib, "--include", INCLUDE,
              "--cuda-include", CUDA_INCLUDE, "--cublas-include", CUDA_INCLUDE,
              "--crt-include", CUDA_INCLUDE, "--cccl-include", CUDA_INCLUDE,
              "--generator", "Ninja", "--configuration", "Release",
              "--binary-root", tmp_path])
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
@pytest.mark.parametrize("mode", ["", "--missing-members", "--wrong-version"])
def test_reference_facade_unit_tests(tmp_path, mode):
    src = _need("tests", "unit", "cuda_compat_facade_tests.cpp")
    exe = tmp_path / "facade_tests"
    b = _run(["g++", "-std=c++20", "-Wall", "-Wextra", "-Wpedantic", "-Werror", "-I", INCLUDE,
              "-isystem", CUDA_INCLUDE, src, "-o", exe, "-pthread"])
    assert b.returncode == 0, b.stderr
    r = _run([exe] + ([mode] if mode else []))
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_reference_package_consumer_runs(tmp_path):
    src = _need("tests", "package_consumer", "cuda_compat.c")
    lib = _lib("compat")
    exe = tmp_path / "cuda_compat_consumer"
    b = _run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", INCLUDE, src, "-o", exe,
              "-L", lib.parent, f"-l:{lib.name}", f"-Wl,-rpath,{lib.parent}"])
    assert b.returncode == 0, b.stderr
    r = _run([exe])
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_reference_preview_gemm_builds_and_prints_usage(tmp_path):
    src = _need("examples", "preview-gemm", "main.cpp")
    lib = _lib("compat")
    exe = tmp_path / "xvram-preview-gemm"
    b = _run(["g++", "-std=c++20", "-Wall", "-Wextra", "-Werror", "-I", INCLUDE, src, "-o", exe,
              "-L", lib.parent, f"-l:{lib.name}", f"-Wl,-rpath,{lib.parent}"])
    assert b.returncode == 0, b.stderr
    r = _run([exe])
    assert r.returncode == 0 and "--run" in r.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_facade_header_rejects_device_compilation(tmp_path):
    """Compiled as CUDA device code the facade stops with its named diagnostic."""
    src = tmp_path / "dev.cpp"
    src.write_text("#define __CUDACC__ 1\n#include <xvram/cuda_compat.hpp>\nint main(){}\n")
    r = _run(["g++", "-std=c++20", "-I", INCLUDE, "-isystem", CUDA_INCLUDE, "-c", src, "-o",
              tmp_path / "dev.o"])
    assert r.returncode != 0 and "XVRAM_CUDA_COMPAT_HOST_ONLY" in r.stderr
