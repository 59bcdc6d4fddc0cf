"""Plain C (and C++) programs drive the two tables through the public headers and the built
libraries, the way the reference's own C consumers do:
  * tests/c_consumer/compat_consumer.c against libxvram_cuda_compat.so: allocate, copy
    in, SGEMM in all four operations with padded leading dimensions, copy out, check
    against a double sum and check the padding, free, shut down;
  * tests/c_consumer/sdk_consumer.c against libxvram.so (xvram_get_api only): an FP32
    row-major GEMM streamed through a 16 MiB budget and an FP64 GEMM submitted as an
    operation, each checked against a wide sum.
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
