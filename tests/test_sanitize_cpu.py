"""The host side of the library under AddressSanitizer with UndefinedBehaviorSanitizer
(leak detection on), and under ThreadSanitizer, over the host-memory fake device (no CUDA):
  * tests/sanitize/runtime_sanitize.cpp drives the residency runtime, planner and
    validation: synchronous and deferred (column-block) in-place GEMMs in all four
    operations, a streamed GEMM with eviction and write-back, a transaction, prefetch,
    releases, and the live budget's sampler thread;
  * tests/sanitize/sdk_sanitize.cpp drives the SDK v1 table on top: a session's worker
    thread, GEMM plans run in place and streamed, operations submitted, polled, waited
    and cancelled, a transaction callback and a prefetch.
The reference's CI runs its host code under the first two sanitizers."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "xvram_b200" / "csrc"
COMMON = [CSRC / "runtime.cpp", CSRC / "planner.cpp", CSRC / "validate.cpp",
          CSRC / "host_util.cpp", ROOT / "tests" / "fake_device" / "fake_device.cpp"]
PROGRAMS = {
    "runtime": COMMON + [ROOT / "tests" / "sanitize" / "runtime_sanitize.cpp"],
    "sdk": COMMON + [CSRC / "sdk_api.cpp", ROOT / "tests" / "sanitize" / "sdk_sanitize.cpp"],
}
SANITIZERS = {
    "address+undefined": ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"],
    "thread": ["-fsanitize=thread"],
}


@pytest.mark.parametrize("program", sorted(PROGRAMS))
@pytest.mark.parametrize("sanitizer", sorted(SANITIZERS))
def test_host_code_under_sanitizers(tmp_path, program, sanitizer):
    if shutil.which("g++") is None:
        pytest.skip("needs g++")
    exe = tmp_path / f"{program}_sanitize"
    build = subprocess.run(
        ["g++", "-std=c++20", "-O1", "-g", *SANITIZERS[sanitizer], "-fno-omit-frame-pointer",
         "-I", str(ROOT / "include"), "-I", str(CSRC), *map(str, PROGRAMS[program]),
         "-lpthread", "-o", str(exe)],
        capture_output=True, text=True)
    if build.returncode != 0 and "san" in build.stderr.lower():
        pytest.skip("the sanitizer runtimes are not installed")
    assert build.returncode == 0, build.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0",
               UBSAN_OPTIONS="print_stacktrace=1", TSAN_OPTIONS="halt_on_error=1")
    # ThreadSanitizer runs the loops about ten times slower: a shorter K for the runtime run
    args = ["quick"] if (sanitizer == "thread" and program == "runtime") else []
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-6000:]
    assert "ok (0 failures)" in r.stdout
