"""The native library loads without a GPU and exports every symbol include/*.h declares."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        # function declarations: an API macro, return type, XVRAM_CALL, then the name
        names |= set(re.findall(r"XVRAM_CALL\s*\n?\s*(xvram_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    from xvram_b200 import _native
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1].split("@")[0] for line in out.splitlines() if " T " in line}
    declared = declared_symbols()
    assert declared, "no declarations found"
    assert declared <= exported, declared - exported
    assert set(_native.EXPORTED) == declared
    # nothing else leaks out of the library
    assert {s for s in exported if not s.startswith("xvram_")} == set()


def test_sdk_library_exports_only_xvram_get_api():
    """libxvram.so is the SDK drop-in: like the reference's SDK library it exports
    xvram_get_api alone, under the version node XVRAM_0.1."""
    from xvram_b200 import _native
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.SDK_LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == {"xvram_get_api@@XVRAM_0.1"}, exported


def test_library_has_no_cuda_runtime_dependency():
    from xvram_b200 import _native
    out = subprocess.run(["ldd", str(_native.LIB_PATH)], capture_output=True, text=True).stdout
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
