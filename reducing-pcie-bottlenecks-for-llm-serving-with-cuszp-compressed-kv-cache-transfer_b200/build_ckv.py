"""Build libckv.so (the sm_100a codec behind include/ckv.h) in-tree.

    python build_ckv.py [--force] [--verbose]

Output: lib/libckv.so next to this file.  The library is self-contained
(static CUDA runtime) and is loaded by cuszp_wrapper_cpp.py through ctypes.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "lib" / "libckv.so"
SOURCES = ["ckv_api.cu", "ckv_encode.cu", "ckv_decode.cu", "ckv_pack.cu", "ckv_noalloc.cu",
           "ckv_int8.cu"]
HEADERS = ["ckv_device.cuh", "ckv_launch.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "ckv.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    # -fmad=false: no multiply/add pair may be contracted into an FMA (the
    # reference rounds its quantiser's and dequantiser's operations
    # separately).  Intended FMAs are explicit fma intrinsics, which the flag
    # does not touch.
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
           "-I", str(ROOT / "include"), "-I", str(CSRC)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(CSRC / s) for s in SOURCES] + ["-o", str(LIB)]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
