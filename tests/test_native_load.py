"""The native library loads without a GPU and exports every symbol include/ declares; the
two drop-in libraries export exactly what the reference's libraries do."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").rglob("*.h"):
        text = h.read_text()
        # function declarations: an API macro, return type, XVRAM_CALL, then the name
        names |= set(re.findall(r"XVRAM_CALL\s*\n?\s*(xvram_[a-z0-9_]+)\s*\(", text))
    return names


def _exports(path: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_every_declared_symbol():
    """libxvram_b200.so exports exactly the declarations of include/, each at its
    version node; the test-only fake-device seam is not among them."""
    from xvram_b200 import _native
    exported = _exports(_native.PRODUCT_LIB_PATH)
    names = {s.split("@")[0] for s in exported}
    declared = declared_symbols()
    assert declared, "no declarations found"
    assert names == declared, names ^ declared
    assert set(_native.EXPORTED) == declared
    assert "xvram_b200_test_set_device_factory" not in names
    nodes = {s.split("@@")[0]: s.split("@@")[1] for s in exported}
    assert nodes.pop("xvram_cuda_compat_get_api") == "XVRAM_CUDA_COMPAT_1.0"
    assert nodes.pop("xvram_get_api") == "XVRAM_0.1"
    assert set(nodes.values()) == {"XVRAM_B200_1.0"}


def test_compat_library_exports_only_the_compat_table():
    """libxvram_cuda_compat.so is the compat drop-in: like the reference's compat library
    (cmake/cuda_compat.exports.map) it exports xvram_cuda_compat_get_api alone, under the
    version node XVRAM_CUDA_COMPAT_1.0."""
    from xvram_b200 import _native
    assert _exports(_native.COMPAT_LIB_PATH) == {
        "xvram_cuda_compat_get_api@@XVRAM_CUDA_COMPAT_1.0"}


def test_sdk_library_exports_only_xvram_get_api():
    """libxvram.so is the SDK drop-in: like the reference's SDK library it exports
    xvram_get_api alone, under the version node XVRAM_0.1."""
    from xvram_b200 import _native
    exported = _exports(_native.SDK_LIB_PATH)
    assert exported == {"xvram_get_api@@XVRAM_0.1"}, exported


def test_library_has_no_cuda_runtime_dependency():
    from xvram_b200 import _native
    for path in (_native.PRODUCT_LIB_PATH, _native.COMPAT_LIB_PATH, _native.SDK_LIB_PATH):
        out = subprocess.run(["ldd", str(path)], capture_output=True, text=True).stdout
        assert "libcudart" not in out  # static runtime; only the driver is needed at run time


def test_get_api_contract_without_gpu():
    import ctypes as C
    from xvram_b200 import compat as cp
    from xvram_b200._native import lib
    st, table = cp.get_api()
    assert st == cp.SUCCESS
    assert table.struct_size == C.sizeof(cp.ApiTable) and table.abi_version == 1
    assert lib.xvram_cuda_compat_get_api(1, C.sizeof(cp.ApiTable), None) == cp.INVALID_ARGUMENT
    assert cp.get_api(version=99)[0] == cp.INCOMPATIBLE_ABI
    assert cp.get_api(size=C.sizeof(cp.ApiTable) - 8)[0] == cp.INCOMPATIBLE_ABI
    for name in cp.FN_TYPES:
        assert getattr(table, name), name


def test_tile_shape_choice_without_a_gpu():
    """xvram_b200_sgemm_tile_shape on a host without a device assumes a 148-SM B200: 192 x 192
    tiles where their waves cost less than 128 x 256 tiles' at 0.95 of the FMA rate, 128 x 128
    for N <= 128, and INVALID_ARGUMENT for sizes outside [1, INT32_MAX] or null outputs."""
    import ctypes as C
    from xvram_b200 import device
    from xvram_b200._native import lib
    assert device.tile_shape(8192, 6144) == (192, 192)      # C2: 9.5 against 10.5 / 0.95 waves
    assert device.tile_shape(9216, 9216) == (192, 192)
    assert device.tile_shape(2560, 2048) == (128, 256)      # 1.5 against 1.08 / 0.95 waves
    assert device.tile_shape(8192, 512) == (128, 256)       # 512 = 2 x 256, 2.67 x 192
    assert device.tile_shape(4096, 100) == (128, 128)
    assert device.tile_shape(100, 4096) == (128, 256)       # M <= 128: 8 warps
    tm, tn = C.c_int32(0), C.c_int32(0)
    for m, n in ((0, 5), (5, 0), (1 << 31, 5), (-1, 5)):
        assert lib.xvram_b200_sgemm_tile_shape(m, n, C.byref(tm), C.byref(tn)) == 1
    assert lib.xvram_b200_sgemm_tile_shape(5, 5, None, C.byref(tn)) == 1
