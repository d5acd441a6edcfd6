"""Build recipe for the test oracles (test infrastructure only).

* ``oracle/_build/libckv_oracle.so`` -- the C restatement in fixed_codec.c,
  built with gcc (-ffp-contract=off, no fast-math).
* ``oracle/_ref/libref_fixed.so`` -- the reference's own
  ``integration/cuszp_wrapper/cuszp_batched_fixed.cu``, compiled unchanged
  from where it lies under the reference checkout, with the two-constant
  stand-in headers in ``oracle/ref_shim`` and the host driver
  ``oracle/ref_driver.cu``.  Built only where the reference checkout exists;
  the .so then travels with the tree.

Neither library is part of the product; only tests/, the smoke check and
bench.py's baseline legs load them.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libckv_oracle.so"
REF_SO = HERE / "_ref" / "libref_fixed.so"
REFERENCE_ROOT = Path(os.environ.get("CKV_REFERENCE_ROOT", "/root/reference"))
REF_KERNEL = REFERENCE_ROOT / "integration" / "cuszp_wrapper" / "cuszp_batched_fixed.cu"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources if s.exists())


def build_oracle(force: bool = False) -> Path:
    src = HERE / "fixed_codec.c"
    if force or _stale(ORACLE_SO, [src, Path(__file__)]):
        ORACLE_SO.parent.mkdir(parents=True, exist_ok=True)
        cmd = [
            "gcc", "-O2", "-std=c11", "-fPIC", "-shared",
            "-ffp-contract=off", "-fno-fast-math", "-pthread",
            str(src), "-o", str(ORACLE_SO), "-lm",
        ]
        subprocess.run(cmd, check=True)
    return ORACLE_SO


def reference_available() -> bool:
    return REF_KERNEL.exists()


def build_ref(force: bool = False) -> Path | None:
    """Compile the reference kernels; returns None where the checkout is absent."""
    if not reference_available():
        return REF_SO if REF_SO.exists() else None
    driver = HERE / "ref_driver.cu"
    shim = HERE / "ref_shim"
    deps = [REF_KERNEL, driver, shim / "cuSZp.h",
            shim / "cuSZp" / "cuSZp_kernels_1D_f32.h", Path(__file__)]
    if force or _stale(REF_SO, deps):
        REF_SO.parent.mkdir(parents=True, exist_ok=True)
        # Default nvcc code generation (no fast-math, fmad as nvcc defaults),
        # as the reference's CMake build leaves CUDA flags at their defaults.
        cmd = [
            NVCC, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
            "-Xcompiler", "-fPIC", "-shared", "-I", str(shim),
            str(REF_KERNEL), str(driver), "-o", str(REF_SO),
        ]
        subprocess.run(cmd, check=True)
    return REF_SO


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
