"""ctypes binding of libckv (include/ckv.h).

Loads lib/libckv.so from this directory, building it with nvcc if it is
missing or older than its sources.  There is no fallback: if the library
cannot be built or loaded, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent

c_size = C.c_size_t
c_float = C.c_float
c_int = C.c_int
c_void_p = C.c_void_p
c_status = C.c_int

CKV_OK = 0
ERRORS = {
    1: "invalid argument",
    2: "unsupported configuration",
    3: "CUDA error",
    4: "compressed data larger than its buffer",
    5: "corrupt or truncated bitstream",
    6: "device-side consistency check failed",
}

DIM_1D, DIM_2D, DIM_3D = 0, 1, 2
MODE_FIXED, MODE_PLAIN, MODE_OUTLIER = 0, 1, 2
TYPE_FLOAT, TYPE_DOUBLE = 0, 1

EXPORTS = (
    "ckv_create", "ckv_destroy", "ckv_get_config", "ckv_update_config",
    "ckv_last_error", "ckv_estimate_compressed_buffer_size",
    "ckv_max_compressed_size", "ckv_compress", "ckv_compress_batch_fixed",
    "ckv_compress_batch_fixed_bf16", "ckv_compress_batch_fixed_bf16_indexed",
    "ckv_compress_batch_fixed_bf16_indexed_groups", "ckv_decompress",
    "ckv_decompress_batch", "ckv_decompress_batch_fixed_bf16",
    "ckv_decompress_batch_fixed_bf16_scatter",
    "ckv_decompress_batch_fixed_bf16_indexed_scatter", "ckv_set_zero_fill",
    "ckv_device_status", "ckv_kernel_launches", "ckv_pack",
    "ckv_set_kernel_timing", "ckv_kernel_time", "ckv_compress_batch_fixed_bf16_noalloc",
    "ckv_pipe_create", "ckv_pipe_destroy", "ckv_pipe_store_bf16", "ckv_pipe_restore_bf16",
    "ckv_pipe_join", "ckv_pipe_record", "ckv_pipe_wait", "ckv_pipe_done", "ckv_pipe_host_capacity",
    "ckv_pipe_store_int8", "ckv_pipe_restore_int8", "ckv_pipe_store_raw", "ckv_pipe_restore_raw",
    "ckv_pipe_host_capacity_int8", "ckv_pipe_host_capacity_raw",
    "ckv_pipe_store_bf16_groups", "ckv_pipe_restore_bf16_groups", "ckv_pipe_host_capacity_groups",
    "ckv_unit_status", "ckv_test_withhold_exchange", "ckv_set_encoder",
)


class Config(C.Structure):
    _fields_ = [
        ("error_bound", c_float),
        ("use_relative_error", c_int),
        ("processing_dim", c_int),
        ("encoding_mode", c_int),
        ("data_type", c_int),
    ]


_lock = threading.Lock()
_lib: C.CDLL | None = None


def library_path() -> Path:
    return HERE / "lib" / "libckv.so"


def _declare(lib: C.CDLL) -> None:
    P = c_void_p
    sig = {
        "ckv_create": (c_status, [C.POINTER(Config), c_int, C.POINTER(c_void_p)]),
        "ckv_destroy": (None, [P]),
        "ckv_get_config": (c_status, [P, C.POINTER(Config)]),
        "ckv_update_config": (c_status, [P, C.POINTER(Config)]),
        "ckv_last_error": (C.c_char_p, [P]),
        "ckv_estimate_compressed_buffer_size": (c_size, [c_size]),
        "ckv_max_compressed_size": (c_size, [c_size]),
        "ckv_compress": (c_status, [P, P, c_size, P, c_size, c_float, P, P, P]),
        "ckv_compress_batch_fixed": (c_status, [P, P, P, P, c_size, c_size, c_size, P, P, P]),
        "ckv_compress_batch_fixed_bf16": (c_status, [P, P, P, P, c_size, c_size, c_size, P, P, P]),
        "ckv_compress_batch_fixed_bf16_indexed": (
            c_status, [P, P, P, P, c_size, c_size, c_size, c_size, P, c_size, c_size, P, P, P]),
        "ckv_compress_batch_fixed_bf16_indexed_groups": (
            c_status, [P, P, P, P, P, P, c_size, c_size, c_size, c_size, P, c_size, P, P, P, P]),
        "ckv_decompress": (c_status, [P, P, c_size, P, c_size, c_float, P]),
        "ckv_decompress_batch": (c_status, [P, P, P, P, P, P, c_size, P]),
        "ckv_decompress_batch_fixed_bf16": (
            c_status, [P, P, P, c_size, P, c_size, c_size, P, P]),
        "ckv_decompress_batch_fixed_bf16_scatter": (
            c_status, [P, P, P, c_size, P, c_size, c_size, c_size, c_size, P, P]),
        "ckv_decompress_batch_fixed_bf16_indexed_scatter": (
            c_status, [P, P, P, c_size, P, P, c_size, c_size, c_size, c_size, P, P]),
        "ckv_set_zero_fill": (c_status, [P, c_int]),
        "ckv_device_status": (c_status, [P, P, c_int, C.POINTER(C.c_uint32)]),
        "ckv_kernel_launches": (C.c_uint64, []),
        "ckv_pack": (c_status, [P, P, P, c_size, P, c_size, c_size, P, P, P]),
        "ckv_set_kernel_timing": (c_status, [P, c_int]),
        "ckv_kernel_time": (c_status, [P, c_int, C.POINTER(c_float)]),
        "ckv_compress_batch_fixed_bf16_noalloc": (
            c_status, [P, P, P, c_size, c_size, c_size, c_float, c_int, P, P, P]),
        "ckv_pipe_create": (c_status, [P, c_size, C.POINTER(c_void_p)]),
        "ckv_pipe_destroy": (None, [P]),
        "ckv_pipe_store_bf16": (
            c_status, [P, P, P, c_size, c_size, P, c_size, P, P, P, P, C.c_uint64, P, P]),
        "ckv_pipe_restore_bf16": (
            c_status, [P, P, P, P, P, c_size, c_size, P, C.c_uint64, P, P]),
        "ckv_pipe_join": (c_status, [P, C.c_uint64, P]),
        "ckv_pipe_record": (c_status, [P, P, P]),
        "ckv_pipe_wait": (c_status, [P, C.c_uint64]),
        "ckv_pipe_done": (c_int, [P, C.c_uint64]),
        "ckv_pipe_host_capacity": (c_size, [c_size, c_size]),
        "ckv_pipe_store_int8": (c_status, [P, P, c_size, c_size, P, c_size, P, P, P, C.c_uint64,
                                           P, P]),
        "ckv_pipe_restore_int8": (c_status, [P, P, P, c_size, c_size, P, C.c_uint64, P, P]),
        "ckv_pipe_store_raw": (c_status, [P, P, c_size, c_size, P, c_size, P, P, C.c_uint64, P,
                                          P]),
        "ckv_pipe_restore_raw": (c_status, [P, P, P, c_size, c_size, P, C.c_uint64, P, P]),
        "ckv_pipe_host_capacity_int8": (c_size, [c_size, c_size]),
        "ckv_pipe_host_capacity_raw": (c_size, [c_size, c_size]),
        "ckv_pipe_store_bf16_groups": (c_status, [P, P, c_size, P, P, c_size, c_size, c_size, c_size,
                                                  P, P, c_size, P, P, P, P, C.c_uint64, P, P]),
        "ckv_pipe_restore_bf16_groups": (c_status, [P, P, P, P, P, c_size, P, P, c_size, c_size,
                                                    c_size, c_size, P, C.c_uint64, P, P]),
        "ckv_pipe_host_capacity_groups": (c_size, [c_size, P, c_size, c_size, c_size]),
        "ckv_unit_status": (c_status, [P, c_size, C.POINTER(C.c_uint32)]),
        "ckv_test_withhold_exchange": (c_status, [P, C.c_uint32, C.c_uint32]),
        "ckv_set_encoder": (c_status, [P, c_int]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load(build: bool = True) -> C.CDLL:
    """The loaded libckv; builds it in-tree first when needed."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build:
            import importlib.util

            spec = importlib.util.spec_from_file_location("build_ckv", HERE / "build_ckv.py")
            builder = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(builder)
            builder.build()
        path = library_path()
        if not path.exists():
            raise ImportError(f"libckv is not built: {path}")
        lib = C.CDLL(str(path))
        _declare(lib)
        _lib = lib
        return lib


def error_message(lib: C.CDLL, ctx, code: int) -> str:
    msg = lib.ckv_last_error(ctx)
    text = msg.decode() if msg else ""
    return text or ERRORS.get(code, f"status {code}")


def ptr_array(ptrs) -> C.Array:
    return (c_void_p * len(ptrs))(*ptrs)


def size_array(values) -> C.Array:
    return (c_size * len(values))(*values)


def float_array(values) -> C.Array:
    return (c_float * len(values))(*values)
