"""Builds and installs the host-memory fake device (tests/fake_device/fake_device.cpp).

Test infrastructure: compiles the fake with g++ into tests/_build, loads it, and installs
its factory into the library with xvram_b200_test_set_device_factory, so sessions and the
compat adapter run the real runtime on host memory without a GPU.

The product libraries do not export that seam.  The CPU suite therefore binds its own
link of the same objects, tests/_build/libxvram_b200_testing.so (testing_library()),
through XVRAM_B200_LIBRARY; tests/conftest.py arranges that for every run that is not
`-m gpu`."""
from __future__ import annotations

import contextlib
import ctypes as C
import subprocess
from pathlib import Path

TESTS = Path(__file__).resolve().parent
ROOT = TESTS.parent
SRC = TESTS / "fake_device" / "fake_device.cpp"
OUT = TESTS / "_build" / "libxvram_fake_device.so"
TESTING_LIB = TESTS / "_build" / "libxvram_b200_testing.so"


def testing_library() -> Path:
    """Links (if stale) the library objects with the seam exported, and returns the path."""
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    from xvram_b200 import build as b
    b.build()
    return b.link(TESTING_LIB, TESTS / "fake_device" / "testing.exports.map")


def build() -> C.CDLL:
    headers = list((ROOT / "xvram_b200" / "csrc").glob("*.hpp")) + list((ROOT / "include").glob("*.h"))
    newest = max([SRC.stat().st_mtime] + [h.stat().st_mtime for h in headers])
    if not OUT.exists() or OUT.stat().st_mtime < newest:
        OUT.parent.mkdir(exist_ok=True)
        subprocess.run(["g++", "-std=c++20", "-O3", "-march=native", "-fPIC", "-shared", f"-I{ROOT / 'include'}",
                        f"-I{ROOT / 'xvram_b200' / 'csrc'}", str(SRC), "-o", str(OUT)],
                       check=True, capture_output=True)
    lib = C.CDLL(str(OUT))
    lib.fake_device_create.restype = C.c_void_p
    lib.fake_device_set_memory.argtypes = [C.c_uint64, C.c_uint64]
    lib.fake_device_fail.argtypes = [C.c_char_p, C.c_long]
    lib.fake_device_set_workspace_fn.argtypes = [C.c_void_p]
    lib.fake_device_set_sm_count.argtypes = [C.c_int]
    lib.fake_device_set_kernel_word.argtypes = [C.c_uint32]
    lib.fake_device_gemm_calls.restype = C.c_uint64
    lib.fake_device_prepares.restype = C.c_uint64
    return lib


@contextlib.contextmanager
def installed(free_bytes: int = 8 << 30, total_bytes: int = 16 << 30):
    """Within the block, new sessions (and a new compat adapter) use the fake device."""
    import pytest
    from xvram_b200._native import has_test_seam, lib
    if not has_test_seam(lib):
        pytest.skip("needs the test link of the library (XVRAM_B200_LIBRARY, tests/conftest.py)")
    fake = build()
    fake.fake_device_set_memory(free_bytes, total_bytes)
    fake.fake_device_fail(b"", -1)
    fake.fake_device_set_sm_count(148)
    fake.fake_device_set_kernel_word(0)
    fake.fake_device_set_workspace_fn(C.cast(lib.xvram_b200_gemm_typed_workspace_bytes,
                                             C.c_void_p))
    factory = C.cast(fake.fake_device_create, C.c_void_p)
    assert lib.xvram_b200_test_set_device_factory(factory) == 0
    try:
        yield fake
    finally:
        lib.xvram_b200_test_set_device_factory(None)
        fake.fake_device_fail(b"", -1)
