"""Plain C (and C++) programs drive the two tables through the public headers and the built
libraries, the way the reference's own C consumers do:
  * tests/c_consumer/compat_consumer.c against libxvram_cuda_compat.so: allocate, copy
    in, SGEMM in all four operations with padded leading dimensions, copy out, check
    against a double sum and check the padding, free, shut down;
  * tests/c_consumer/sdk_consumer.c against libxvram.so (xvram_get_api only): an FP32
    row-major GEMM streamed through a 16 MiB budget and an FP64 GEMM submitted as an
    operation, each checked against a wide sum;
  * tests/c_consumer/facade_consumer.cpp against libxvram_cuda_compat.so through the C++
    facade <xvram/cuda_compat.hpp>: a program written with cudaMalloc / cudaMemcpy /
    cublasSgemm spellings, with no CUDA runtime or cuBLAS linked;
  * the reference's own examples/preview-gemm program, built against this library by
    tests/ref_consumers/Makefile (the reference tree is not on GPU machines, so the
    program is built beforehand and travels with the libraries).
Building and linking needs no GPU; running does."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c_consumer"
LIB = ROOT / "xvram_b200" / "lib"
PROGRAMS = {"compat": ("compat_consumer.c", "xvram_cuda_compat"), "sdk": ("sdk_consumer.c", "xvram")}
CUDA_INCLUDE = Path("/usr/local/cuda/include")
PREVIEW_GEMM = ROOT / "tests" / "_build" / "ref_consumers" / "xvram-preview-gemm"


def build(tmp_path: Path, cc: str, program: str) -> Path:
    if shutil.which(cc) is None:
        pytest.skip(f"needs {cc}")
    src, lib = PROGRAMS[program]
    exe = tmp_path / f"{program}_{cc}"
    lang, std = ("c", "-std=c11") if cc == "gcc" else ("c++", "-std=c++17")
    subprocess.run([cc, "-x", lang, std, "-O2", "-Wall", "-Wextra", "-Werror",
                    "-I", str(ROOT / "include"), str(SRC / src), "-L", str(LIB), f"-l{lib}",
                    f"-Wl,-rpath,{LIB}", "-lm", "-o", str(exe)], check=True)
    return exe


def build_facade(tmp_path: Path) -> Path:
    if shutil.which("g++") is None or not (CUDA_INCLUDE / "cublas_v2.h").exists():
        pytest.skip("needs g++ and the CUDA toolkit headers")
    exe = tmp_path / "facade_consumer"
    subprocess.run(["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-Wpedantic", "-Werror",
                    "-I", str(ROOT / "include"), "-isystem", str(CUDA_INCLUDE),
                    str(SRC / "facade_consumer.cpp"), "-L", str(LIB), "-l:libxvram_cuda_compat.so",
                    f"-Wl,-rpath,{LIB}", "-o", str(exe)], check=True)
    return exe


def test_facade_consumer_builds_without_cuda_libraries(tmp_path):
    exe = build_facade(tmp_path)
    out = subprocess.run(["ldd", str(exe)], capture_output=True, text=True).stdout
    assert "libxvram_cuda_compat.so" in out
    assert "libcudart" not in out and "libcublas" not in out


@pytest.mark.gpu
def test_facade_consumer_runs_cublas_spelled_sgemm(tmp_path):
    exe = build_facade(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 mismatches" in r.stdout and "facade consumer passed" in r.stdout


@pytest.mark.gpu
def test_reference_preview_gemm_example_passes():
    """The reference's own example program, unchanged, on this library: it initialises the
    adapter, runs a 37 x 19 x 67 SGEMM, checks it against its CPU FP64 sum and shuts down."""
    if not PREVIEW_GEMM.exists():
        pytest.skip("tests/_build/ref_consumers not built (needs the reference tree at build time)")
    r = subprocess.run([str(PREVIEW_GEMM), "--run"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS: small integration example; cleanup completed." in r.stdout


@pytest.mark.parametrize("program", sorted(PROGRAMS))
@pytest.mark.parametrize("cc", ["gcc", "g++"])
def test_consumer_builds_and_links(tmp_path, cc, program):
    assert build(tmp_path, cc, program).exists()


@pytest.mark.gpu
@pytest.mark.parametrize("cc", ["gcc", "g++"])
def test_compat_consumer_runs_all_operations(tmp_path, cc):
    exe = build(tmp_path, cc, "compat")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    for op in ("NN", "NT", "TN", "TT"):
        assert f"op {op}: 0 mismatches" in r.stdout


@pytest.mark.gpu
def test_sdk_consumer_streams_and_submits(tmp_path):
    exe = build(tmp_path, "gcc", "sdk")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fp32 row-major streamed" in r.stdout and "0 mismatches" in r.stdout
