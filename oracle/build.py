"""Build recipe for the test oracles (test infrastructure only).

* ``oracle/_build/libckv_oracle.so`` -- the C restatement in fixed_codec.c,
  built with gcc (-ffp-contract=off, no fast-math).
* ``oracle/_ref/libref_fixed.so`` -- the reference's own
  ``integration/cuszp_wrapper/cuszp_batched_fixed.cu``, compiled unchanged
  from where it lies under the reference checkout, with the two-constant
  stand-in headers in ``oracle/ref_shim`` and the host driver
  ``oracle/ref_driver.cu``.
* ``oracle/_ref/py/`` -- the reference's vLLM connector
  (``integration/compression_pipeline/*.py``) and its connector tests
  (``tests/test_vllm_v1_compressed_offload.py``), byte-compiled unchanged
  from where they lie (``.pyc`` only, no source copied).  The drop-in test
  (tests/test_reference_connector_gpu.py) runs those tests with this
  repository's ``cuszp_wrapper_cpp`` in place of the reference's binding.

Both are built only where a reference checkout exists and then travel with
the tree (``oracle/_ref`` is kept out of version control).  The checkout is
``$CKV_REFERENCE_ROOT`` when set, else a sibling directory named
``reference`` next to this repository.

Nothing here is part of the product; only tests/, the smoke check and
bench.py's baseline legs load it.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libckv_oracle.so"
REF_SO = HERE / "_ref" / "libref_fixed.so"
REF_PY = HERE / "_ref" / "py"
_env_root = os.environ.get("CKV_REFERENCE_ROOT")
REFERENCE_ROOT = Path(_env_root) if _env_root else HERE.parent.parent / "reference"
REF_KERNEL = REFERENCE_ROOT / "integration" / "cuszp_wrapper" / "cuszp_batched_fixed.cu"
# reference module -> its byte-compiled place under REF_PY (".refpyc": the
# tree is copied to the GPU box without *.pyc files, and nothing imports
# these by accident; tests load them through an explicit finder)
CONNECTOR_MODULES = {
    "integration/compression_pipeline/vllm_v1_compressed_offload.py":
        "integration/compression_pipeline/vllm_v1_compressed_offload.refpyc",
    "integration/compression_pipeline/native_lossless.py":
        "integration/compression_pipeline/native_lossless.refpyc",
    "tests/test_vllm_v1_compressed_offload.py": "ref_tests/test_vllm_v1_compressed_offload.refpyc",
}
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


def stage_connector(force: bool = False) -> Path | None:
    """Byte-compile the reference's connector and its tests into REF_PY.

    The compiled modules load without their sources (tests use Python's
    sourceless loader on them), so the GPU box, which has no reference
    checkout, can still run the unmodified connector.  Returns REF_PY, or
    None where neither the checkout nor an earlier staging exists."""
    import py_compile

    sources = {REFERENCE_ROOT / src: REF_PY / dst for src, dst in CONNECTOR_MODULES.items()}
    if not all(src.exists() for src in sources):
        staged = all(dst.exists() for dst in sources.values())
        return REF_PY if staged else None
    for src, dst in sources.items():
        if force or _stale(dst, [src, Path(__file__)]):
            dst.parent.mkdir(parents=True, exist_ok=True)
            py_compile.compile(str(src), cfile=str(dst), doraise=True,
                               invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    return REF_PY


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
    print(stage_connector(force="--force" in sys.argv))
