"""The public headers and the ctypes mirrors are layout-identical to the reference ABI.

tests/golden/abi_layout.json was produced from the reference's include/xvram headers by
tests/golden/make_abi_layout.py (sizeof/offsetof of every field, enumerator values and
the default-initialiser bytes)."""
from __future__ import annotations

import ctypes as C
import json
import shutil
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _golden():
    return json.loads((HERE / "golden" / "abi_layout.json").read_text())


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_headers_match_reference_layout():
    import sys
    sys.path.insert(0, str(HERE / "golden"))
    import make_abi_layout
    mine = make_abi_layout.dump(["-I", str(ROOT / "include")], [])
    want = _golden()
    assert set(mine) == set(want)
    diffs = {k: (want[k], mine[k]) for k in want if want[k] != mine[k]}
    assert not diffs


def test_headers_compile_as_c_and_cpp(tmp_path):
    if shutil.which("gcc") is None or shutil.which("g++") is None:
        pytest.skip("needs gcc/g++")
    import subprocess
    src = tmp_path / "consumer.c"
    src.write_text(
        '#include <xvram/cuda_compat.h>\n#include "xvram_b200.h"\n'
        "int main(void){xvram_cuda_compat_config_v1 c = XVRAM_CUDA_COMPAT_CONFIG_V1_INIT;\n"
        "xvram_error_info_v1 e = XVRAM_ERROR_INFO_V1_INIT; (void)e;\n"
        "return c.session.chunk_size_bytes == 67108864u ? 0 : 1;}\n")
    for cc, std in (("gcc", "-std=c11"), ("g++", "-std=c++17")):
        exe = tmp_path / f"a_{cc}"
        subprocess.run([cc, std, "-Wall", "-Werror", "-x", "c" if cc == "gcc" else "c++",
                        "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
        assert subprocess.run([str(exe)]).returncode == 0


def test_ctypes_mirrors_match_reference_layout():
    from xvram_b200 import compat as cp
    want = _golden()
    structs = {
        "xvram_error_info_v1": cp.ErrorInfo,
        "xvram_session_config_v1": cp.SessionConfig,
        "xvram_session_telemetry_v1": cp.SessionTelemetry,
        "xvram_cuda_compat_config_v1": cp.CompatConfig,
        "xvram_cuda_compat_telemetry_v1": cp.CompatTelemetry,
        "xvram_cuda_compat_api_v1": cp.ApiTable,
    }
    for cname, py in structs.items():
        assert C.sizeof(py) == want[f"sizeof {cname}"], cname
        for field, _ in py._fields_:
            off, size = want[f"{cname}.{field}"]
            assert getattr(py, field).offset == off, (cname, field)
            assert getattr(py, field).size == size, (cname, field)


def test_ctypes_default_initialisers_match_macros():
    from xvram_b200 import compat as cp
    want = _golden()
    s = cp.session_config_init()
    assert bytes(s).hex() == want["init xvram_session_config_v1"]
    c = cp.compat_config_init()
    head = want["init xvram_cuda_compat_config_v1[head]"]
    assert bytes(c)[: len(head) // 2].hex() == head
