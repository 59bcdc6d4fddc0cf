"""The residency runtime, planner and validation under AddressSanitizer and
UndefinedBehaviorSanitizer (with leak detection), and under ThreadSanitizer, driven over
the host-memory fake device
by tests/sanitize/runtime_sanitize.cpp: synchronous and deferred (column-block) in-place
GEMMs in all four operations, a streamed GEMM with eviction and write-back, a
transaction, prefetch, releases, and the live budget's sampler thread.  The reference's
CI runs its host code under the same sanitizers."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "xvram_b200" / "csrc"
SOURCES = [CSRC / "runtime.cpp", CSRC / "planner.cpp", CSRC / "validate.cpp",
           CSRC / "host_util.cpp", ROOT / "tests" / "fake_device" / "fake_device.cpp",
           ROOT / "tests" / "sanitize" / "runtime_sanitize.cpp"]


@pytest.mark.parametrize("sanitizers,args", [
    (["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"], []),
    # races between the caller's thread, the budget sampler thread and the copy helpers;
    # K shortened because the loops run about ten times slower
    (["-fsanitize=thread"], ["quick"]),
], ids=["address+undefined", "thread"])
def test_runtime_under_sanitizers(tmp_path, sanitizers, args):
    if shutil.which("g++") is None:
        pytest.skip("needs g++")
    exe = tmp_path / "runtime_sanitize"
    build = subprocess.run(
        ["g++", "-std=c++20", "-O1", "-g", *sanitizers, "-fno-omit-frame-pointer",
         "-I", str(ROOT / "include"), "-I", str(CSRC), *map(str, SOURCES), "-lpthread", "-o",
         str(exe)],
        capture_output=True, text=True)
    if build.returncode != 0 and "san" in build.stderr.lower():
        pytest.skip("the sanitizer runtimes are not installed")
    assert build.returncode == 0, build.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0",
               UBSAN_OPTIONS="print_stacktrace=1", TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-6000:]
    assert "ok (0 failures)" in r.stdout
