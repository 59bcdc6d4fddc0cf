"""Builds the native library xvram_b200/lib/libxvram_cuda_compat.so for sm_100a.

    python -m xvram_b200.build            # incremental
    python -m xvram_b200.build --clean

Every CUDA source is compiled with `-gencode arch=compute_100a,code=sm_100a`; host
sources with g++ -std=c++20.  The library links the CUDA runtime statically and
resolves driver entry points at run time, so it only needs libcuda.so.1 from the
driver on the machine that loads it.
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
LIB = PKG / "lib" / "libxvram_cuda_compat.so"
# The same objects linked as the SDK drop-in: exports xvram_get_api only.
SDK_LIB = PKG / "lib" / "libxvram.so"
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
    hs = list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
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
    newest = max(o.stat().st_mtime for o in objs)
    for lib, script in ((LIB, "exports.map"), (SDK_LIB, "sdk.exports.map")):
        if lib.exists() and lib.stat().st_mtime >= max(newest, (CSRC / script).stat().st_mtime):
            continue
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC",
               f"-Xlinker=--version-script={CSRC / script}", "-Xlinker=--no-undefined",
               *map(str, objs), "-o", str(lib), "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    if a.clean:
        shutil.rmtree(BUILD, ignore_errors=True)
        for lib in (LIB, SDK_LIB):
            if lib.exists():
                lib.unlink()
    print(build(a.verbose))


if __name__ == "__main__":
    main()
