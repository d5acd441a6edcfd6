"""Host-side checks that need no GPU: the C-ABI library loads and exports
every entry point include/ckv.h declares, and the Python module mirrors the
reference's pybind11 surface (pybind11_bindings.cpp:9-264)."""
import ctypes
import inspect
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "ckv.h").read_text()
    return sorted(set(re.findall(r"^CKV_API [^;]*?\b(ckv_\w+)\(", text, re.M)))


def test_header_declares_every_reference_method():
    names = declared_functions()
    for method in ("compress", "compress_batch_fixed", "compress_batch_fixed_bf16",
                   "compress_batch_fixed_bf16_indexed",
                   "compress_batch_fixed_bf16_indexed_groups", "decompress",
                   "decompress_batch", "decompress_batch_fixed_bf16",
                   "decompress_batch_fixed_bf16_scatter",
                   "decompress_batch_fixed_bf16_indexed_scatter",
                   "estimate_compressed_buffer_size", "get_config", "update_config",
                   "create", "destroy"):
        assert f"ckv_{method}" in names


def test_library_exports_every_declared_symbol():
    import _ckv
    lib = _ckv.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(_ckv.EXPORTS) == set(declared_functions())
    raw = ctypes.CDLL(str(_ckv.library_path()))
    for name in declared_functions():
        assert getattr(raw, name)


def test_host_only_entry_points():
    import _ckv
    lib = _ckv.load()
    assert lib.ckv_estimate_compressed_buffer_size(1000) == 2000
    # worst case: header + every block at rate 31 plus sign word
    assert lib.ckv_max_compressed_size(32768) == 1024 + 1024 * 132
    assert lib.ckv_max_compressed_size(32769) == 2048 + 1025 * 132
    assert isinstance(lib.ckv_kernel_launches(), int)
    # pipeline host buffers for cuSZp pages: every unit at its worst case,
    # 16-byte aligned, plus the alignment slack of each unit
    import ctypes as C

    def worst(n):
        nb = (n + 31) // 32
        return ((n + 32767) // 32768 * 1024 + nb * 132 + 15) // 16 * 16

    n = 229376
    assert lib.ckv_pipe_host_capacity(5, n) == 5 * (worst(n) + 16)
    sel = (C.c_size_t * 2)(7, 21)
    cap = lib.ckv_pipe_host_capacity_groups(3, sel, 2, 2, 4096)
    assert cap == 3 * (worst(2 * 7 * 4096) + 16 + worst(2 * 21 * 4096) + 16)
    # INT8 and raw pages have known sizes: their 16-byte strides exactly
    assert lib.ckv_pipe_host_capacity_int8(4, 1001) == 4 * ((1004 + 4 + 15) // 16 * 16)
    assert lib.ckv_pipe_host_capacity_raw(4, 1002) == 4 * ((1002 + 15) // 16 * 16)


def test_python_surface_matches_reference():
    import cuszp_wrapper_cpp as m
    assert [e.name for e in m.CuszpDim] == ["DIM_1D", "DIM_2D", "DIM_3D"]
    assert [e.name for e in m.CuszpMode] == ["MODE_FIXED", "MODE_PLAIN", "MODE_OUTLIER"]
    assert [e.name for e in m.CuszpType] == ["TYPE_FLOAT", "TYPE_DOUBLE"]
    assert m.DIM_1D is m.CuszpDim.DIM_1D and m.MODE_FIXED is m.CuszpMode.MODE_FIXED
    cfg = m.CompressionConfig()
    assert cfg.error_bound == pytest.approx(1e-4) and cfg.use_relative_error
    assert cfg.encoding_mode == m.CuszpMode.MODE_PLAIN
    cfg.error_bound = 1e-5
    assert cfg.error_bound == 1e-5
    expected = {
        "compress": ["input_tensor", "compressed_buffer", "eps_override"],
        "compress_batch_fixed": ["input_tensors", "compressed_buffers", "eps_overrides"],
        "compress_batch_fixed_bf16": ["input_tensors", "compressed_buffers", "eps_overrides"],
        "compress_batch_fixed_bf16_indexed": [
            "input_tensors", "compressed_buffers", "layer_indices", "prefix_count",
            "source_layers", "elements_per_layer", "eps_overrides"],
        "compress_batch_fixed_bf16_indexed_groups": [
            "input_tensors", "compressed_buffers", "layer_indices", "group_sizes",
            "prefix_count", "source_layers", "elements_per_layer", "eps_overrides"],
        "decompress": ["compressed_buffer", "compressed_size", "output_tensor",
                       "actual_error_bound"],
        "decompress_batch": ["compressed_buffers", "compressed_sizes", "output_tensors",
                             "actual_error_bounds"],
        "decompress_batch_fixed_bf16": ["compressed_buffers", "compressed_sizes",
                                        "output_tensor", "num_elements_per_page",
                                        "actual_error_bounds"],
        "decompress_batch_fixed_bf16_scatter": [
            "compressed_buffers", "compressed_sizes", "output_tensors",
            "num_elements_per_page", "destinations_per_page",
            "elements_per_destination", "actual_error_bounds"],
        "decompress_batch_fixed_bf16_indexed_scatter": [
            "compressed_buffers", "compressed_sizes", "output_tensors", "layer_indices",
            "prefix_count", "source_layers", "elements_per_layer", "actual_error_bounds"],
    }
    for name, args in expected.items():
        params = [p for p in inspect.signature(getattr(m.CuSZpWrapper, name)).parameters
                  if p != "self" and not p.startswith("_")]
        assert params == args, name
    assert m.CuSZpWrapper.estimate_compressed_buffer_size(4096) == 8192
    assert inspect.signature(m.CuSZpWrapper.compress).parameters["eps_override"].default == -1.0


def test_enum_values_agree_everywhere():
    """include/ckv.h, the stand-in cuSZp header the reference's kernels are
    built with (oracle/ref_shim/cuSZp.h) and the Python enums give every
    cuszp_dim_t / cuszp_mode_t / cuszp_type_t name the same value, in the
    reference's binding order (pybind11_bindings.cpp:13-28), so a caller that
    passes its configuration's encoding_mode straight through reads FIXED as
    FIXED."""
    import _ckv
    import cuszp_wrapper_cpp as m

    header = (ROOT / "include" / "ckv.h").read_text()
    ckv = {k: int(v) for k, v in re.findall(r"^#define CKV_((?:DIM|MODE|TYPE)_\w+) (\d+)", header, re.M)}
    shim = (ROOT / "oracle" / "ref_shim" / "cuSZp.h").read_text()
    ref = {k: int(v) for k, v in re.findall(r"CUSZP_((?:DIM|MODE|TYPE)_\w+) = (\d+)", shim)}
    assert ckv == ref and len(ckv) == 8
    assert ckv == {"DIM_1D": 0, "DIM_2D": 1, "DIM_3D": 2, "MODE_FIXED": 0, "MODE_PLAIN": 1,
                   "MODE_OUTLIER": 2, "TYPE_FLOAT": 0, "TYPE_DOUBLE": 1}
    for enum in (m.CuszpDim, m.CuszpMode, m.CuszpType):
        for e in enum:
            assert int(e) == ckv[e.name] == getattr(_ckv, e.name), e.name
