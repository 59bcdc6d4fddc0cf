"""Builds the native libraries under xvram_b200/lib for sm_100a.

    python -m xvram_b200.build            # incremental
    python -m xvram_b200.build --clean

One set of objects is linked three times, each with its own export list:

* libxvram_b200.so        the native library (compat table, SDK table, xvram_b200_*);
                          the Python package binds this one.
* libxvram_cuda_compat.so the compat drop-in: exports xvram_cuda_compat_get_api alone,
                          at version node XVRAM_CUDA_COMPAT_1.0, as the reference's does.
* libxvram.so             the SDK drop-in: exports xvram_get_api alone (XVRAM_0.1).

Every CUDA source is compiled with `-gencode arch=compute_100a,code=sm_100a`; host
sources with g++ -std=c++20.  The libraries link the CUDA runtime statically and
resolve driver entry points at run time, so they only need libcuda.so.1 from the
driver on the machine that loads them.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libxvram_b200.so"
COMPAT_LIB = PKG / "lib" / "libxvram_cuda_compat.so"
SDK_LIB = PKG / "lib" / "libxvram.so"
# (library, export map in csrc/)
LINKS = ((LIB, "native.exports.map"), (COMPAT_LIB, "compat.exports.map"),
         (SDK_LIB, "sdk.exports.map"))
INCLUDE = ROOT / "include"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", f"{CUDA_HOME}/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-DXVRAM_BUILDING_CUDA_COMPAT", "-DXVRAM_BUILDING_LIBRARY", f"-I{INCLUDE}",
          f"-I{CSRC}"]


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(CSRC.glob("*.cpp"))
    return cu, cpp


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.rglob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[-1]}")


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    cu, cpp = _sources()
    hdr = _headers_mtime()
    objs = []
    for src in cu + cpp:
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            continue
        if src.suffix == ".cu":
            cmd = [NVCC, *ARCH, "-lineinfo", "-std=c++17", *COMMON, "-Xcompiler",
                   "-fPIC,-fvisibility=hidden", "-c", str(src), "-o", str(obj)]
        else:
            cmd = [CXX, "-std=c++20", *COMMON, f"-I{CUDA_HOME}/include", "-fPIC",
                   "-fvisibility=hidden", "-Wall", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    for lib, script in LINKS:
        link(lib, CSRC / script, objs, verbose)
    return LIB


def objects() -> list[Path]:
    """The compiled objects every library is linked from (after build())."""
    cu, cpp = _sources()
    return [BUILD / (src.name + ".o") for src in cu + cpp]


def link(lib: Path, export_map: Path, objs: list[Path] | None = None,
         verbose: bool = False) -> Path:
    """Links `objs` (default: all objects) into `lib` with the given version script,
    unless `lib` is newer than both."""
    objs = objects() if objs is None else objs
    newest = max(max(o.stat().st_mtime for o in objs), export_map.stat().st_mtime)
    if lib.exists() and lib.stat().st_mtime >= newest:
        return lib
    lib.parent.mkdir(parents=True, exist_ok=True)
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC",
           f"-Xlinker=--version-script={export_map}", "-Xlinker=--no-undefined",
           *map(str, objs), "-o", str(lib), "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd))
    _run(cmd)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    if a.clean:
        shutil.rmtree(BUILD, ignore_errors=True)
        for lib, _ in LINKS:
            if lib.exists():
                lib.unlink()
    print(build(a.verbose))


if __name__ == "__main__":
    main()
