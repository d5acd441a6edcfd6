"""Drop-in replacement for the reference's ``cuszp_wrapper_cpp`` module.

Same names, arguments, defaults, return tuples and error behaviour as the
pybind11 module of integration/cuszp_wrapper/pybind11_bindings.cpp:9-264,
so ``integration/compression_pipeline/vllm_v1_compressed_offload.py`` (which
does ``import cuszp_wrapper_cpp`` after putting its own directory on
sys.path, vllm_v1_compressed_offload.py:41-45) runs on it unchanged when this
directory comes first on sys.path.

Every method validates its tensors the way CuSZpWrapper does
(cuszp_wrapper.cpp) and returns False -- never raises -- when a
precondition fails, then calls libckv (include/ckv.h) with raw device
pointers on the caller's current PyTorch stream (pybind11_bindings.cpp:54).
Errors reported by libckv are printed to stderr, as the reference prints
CUDA errors (cuszp_wrapper.cpp:11-19).

Only the fixed encoding mode is implemented; plain and outlier modes (the
upstream cuSZp Lorenzo / outlier encoders) make compress and decompress
return False with a message.
"""
from __future__ import annotations

import enum
import sys

import torch

import _ckv

_lib = _ckv.load()


class CuszpDim(enum.IntEnum):
    DIM_1D = _ckv.DIM_1D
    DIM_2D = _ckv.DIM_2D
    DIM_3D = _ckv.DIM_3D


class CuszpMode(enum.IntEnum):
    MODE_FIXED = _ckv.MODE_FIXED
    MODE_PLAIN = _ckv.MODE_PLAIN
    MODE_OUTLIER = _ckv.MODE_OUTLIER


class CuszpType(enum.IntEnum):
    TYPE_FLOAT = _ckv.TYPE_FLOAT
    TYPE_DOUBLE = _ckv.TYPE_DOUBLE


# py::enum_<...>.export_values() (pybind11_bindings.cpp:17,23,28)
DIM_1D, DIM_2D, DIM_3D = CuszpDim.DIM_1D, CuszpDim.DIM_2D, CuszpDim.DIM_3D
MODE_FIXED, MODE_PLAIN, MODE_OUTLIER = (
    CuszpMode.MODE_FIXED, CuszpMode.MODE_PLAIN, CuszpMode.MODE_OUTLIER)
TYPE_FLOAT, TYPE_DOUBLE = CuszpType.TYPE_FLOAT, CuszpType.TYPE_DOUBLE


class CompressionConfig:
    """CuSZpWrapper::CompressionConfig (cuszp_wrapper.h:11-17,
    pybind11_bindings.cpp:31-43)."""

    def __init__(self, error_bound: float = 1e-4, use_relative_error: bool = True,
                 processing_dim: CuszpDim = CuszpDim.DIM_1D,
                 encoding_mode: CuszpMode = CuszpMode.MODE_PLAIN,
                 data_type: CuszpType = CuszpType.TYPE_FLOAT):
        self.error_bound = float(error_bound)
        self.use_relative_error = bool(use_relative_error)
        self.processing_dim = CuszpDim(processing_dim)
        self.encoding_mode = CuszpMode(encoding_mode)
        self.data_type = CuszpType(data_type)

    def _as_c(self) -> _ckv.Config:
        return _ckv.Config(float(self.error_bound), int(bool(self.use_relative_error)),
                           int(self.processing_dim), int(self.encoding_mode),
                           int(self.data_type))

    @classmethod
    def _from_c(cls, c: _ckv.Config) -> "CompressionConfig":
        return cls(c.error_bound, bool(c.use_relative_error), CuszpDim(c.processing_dim),
                   CuszpMode(c.encoding_mode), CuszpType(c.data_type))

    def __repr__(self) -> str:
        return (f"CompressionConfig(error_bound={self.error_bound!r}, "
                f"use_relative_error={self.use_relative_error!r}, "
                f"processing_dim={self.processing_dim!r}, "
                f"encoding_mode={self.encoding_mode!r}, data_type={self.data_type!r})")


def _copy_config(c: CompressionConfig) -> CompressionConfig:
    return CompressionConfig(c.error_bound, c.use_relative_error, c.processing_dim,
                             c.encoding_mode, c.data_type)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _report(message: str) -> None:
    print(f"Error: {message}", file=sys.stderr)


class CuSZpWrapper:
    """CuSZpWrapper (cuszp_wrapper.h:9-158) backed by libckv."""

    def __init__(self, config: CompressionConfig, device_id: int = 0):
        # The C++ wrapper keeps its own copy of the config (cuszp_wrapper.h:130).
        self._config = _copy_config(config)
        self._device_id = int(device_id)
        self._device = torch.device("cuda", self._device_id)
        ctx = _ckv.c_void_p()
        cfg = config._as_c()
        status = _lib.ckv_create(cfg, self._device_id, _ckv.C.byref(ctx))
        if status != _ckv.CKV_OK:
            raise RuntimeError(f"libckv context creation failed on device {device_id}")
        self._ctx = ctx

    def __del__(self):
        ctx = getattr(self, "_ctx", None)
        if ctx is not None and ctx.value:
            _lib.ckv_destroy(ctx)
            self._ctx = None

    # -- helpers ---------------------------------------------------------
    def _call(self, fn, *args) -> bool:
        status = fn(self._ctx, *args)
        if status != _ckv.CKV_OK:
            _report(_ckv.error_message(_lib, self._ctx, status))
            return False
        return True

    def _on_device(self, t: torch.Tensor) -> bool:
        return t.is_cuda and t.get_device() == self._device_id

    def _fixed_1d_float(self) -> bool:
        c = self._config
        return (c.processing_dim == CuszpDim.DIM_1D and c.data_type == CuszpType.TYPE_FLOAT
                and c.encoding_mode == CuszpMode.MODE_FIXED)

    def _eps_list(self, eps_overrides, count):
        if eps_overrides is None or len(eps_overrides) == 0:
            return None
        return _ckv.float_array([float(e) for e in eps_overrides])

    # -- compression -----------------------------------------------------
    def compress(self, input_tensor: torch.Tensor, compressed_buffer: torch.Tensor,
                 eps_override: float = -1.0):
        """compress (pybind11_bindings.cpp:49-64; cuszp_wrapper.cpp:216-325).

        Returns (success, buffer, compressed_size, actual_error_bound).  A
        buffer smaller than estimate_compressed_buffer_size(nbytes) is
        replaced by a new one of that size (cuszp_wrapper.cpp:232-240); a
        new buffer is also at least the worst-case compressed size.
        """
        if not input_tensor.is_cuda:
            _report("Input tensor must be on GPU")
            return False, compressed_buffer, 0, 0.0
        if input_tensor.dtype != torch.float32 or not input_tensor.is_contiguous():
            _report("compress expects a contiguous float32 CUDA tensor")
            return False, compressed_buffer, 0, 0.0
        n = input_tensor.numel()
        nbytes = n * input_tensor.element_size()
        estimated = _lib.ckv_estimate_compressed_buffer_size(nbytes)
        capacity = compressed_buffer.numel() * compressed_buffer.element_size()
        if capacity < estimated or not compressed_buffer.is_cuda:
            compressed_buffer = torch.empty(
                max(estimated, _lib.ckv_max_compressed_size(n)), dtype=torch.uint8,
                device=input_tensor.device)
            capacity = compressed_buffer.numel()
        size = _ckv.c_size(0)
        bound = _ckv.c_float(0.0)
        ok = self._call(_lib.ckv_compress, input_tensor.data_ptr(), n,
                        compressed_buffer.data_ptr(), capacity, float(eps_override),
                        _ckv.C.byref(size), _ckv.C.byref(bound),
                        _stream(input_tensor.device))
        return ok, compressed_buffer, int(size.value), float(bound.value)

    def _compress_batch(self, fn, input_tensors, compressed_buffers, eps_overrides, dtype):
        batch = len(input_tensors)
        if (batch == 0 or len(compressed_buffers) != batch
                or (eps_overrides and len(eps_overrides) != batch)
                or not self._fixed_1d_float()):
            return False, [], []
        n = input_tensors[0].numel()
        required = _lib.ckv_estimate_compressed_buffer_size(n * 4)
        for t, o in zip(input_tensors, compressed_buffers):
            if (not self._on_device(t) or not self._on_device(o) or t.dtype != dtype
                    or o.dtype != torch.uint8 or not t.is_contiguous()
                    or not o.is_contiguous() or t.numel() != n or o.numel() < required):
                return False, [], []
        capacity = min(o.numel() for o in compressed_buffers)
        sizes = (_ckv.c_size * batch)()
        bounds = (_ckv.c_float * batch)()
        ok = self._call(fn, _ckv.ptr_array([t.data_ptr() for t in input_tensors]),
                        _ckv.ptr_array([o.data_ptr() for o in compressed_buffers]),
                        self._eps_list(eps_overrides, batch), batch, n, capacity,
                        sizes, bounds, _stream(self._device))
        if not ok:
            return False, [], []
        return True, [int(s) for s in sizes], [float(b) for b in bounds]

    def compress_batch_fixed(self, input_tensors, compressed_buffers, eps_overrides):
        """compress_batch_fixed (pybind11_bindings.cpp:65-82;
        cuszp_wrapper.cpp:327-429): FP32 pages -> (ok, sizes, bounds)."""
        return self._compress_batch(_lib.ckv_compress_batch_fixed, input_tensors,
                                    compressed_buffers, eps_overrides, torch.float32)

    def compress_batch_fixed_bf16(self, input_tensors, compressed_buffers, eps_overrides):
        """compress_batch_fixed_bf16 (pybind11_bindings.cpp:84-101;
        cuszp_wrapper.cpp:431-544): BF16 pages -> (ok, sizes, bounds)."""
        return self._compress_batch(_lib.ckv_compress_batch_fixed_bf16, input_tensors,
                                    compressed_buffers, eps_overrides, torch.bfloat16)

    def _check_layer_index(self, idx: torch.Tensor, source_layers: int) -> bool:
        return (isinstance(idx, torch.Tensor) and idx.numel() > 0
                and idx.numel() <= source_layers and self._on_device(idx)
                and idx.dtype == torch.int64 and idx.is_contiguous())

    def compress_batch_fixed_bf16_indexed(self, input_tensors, compressed_buffers,
                                          layer_indices, prefix_count, source_layers,
                                          elements_per_layer, eps_overrides):
        """compress_batch_fixed_bf16_indexed (pybind11_bindings.cpp:104-132;
        cuszp_wrapper.cpp:548-681)."""
        return self.compress_batch_fixed_bf16_indexed_groups(
            input_tensors, compressed_buffers, [layer_indices], [len(input_tensors)],
            prefix_count, source_layers, elements_per_layer, eps_overrides,
            _checked_single=True)

    def compress_batch_fixed_bf16_indexed_groups(self, input_tensors, compressed_buffers,
                                                 layer_indices, group_sizes, prefix_count,
                                                 source_layers, elements_per_layer,
                                                 eps_overrides, _checked_single=False):
        """compress_batch_fixed_bf16_indexed_groups (pybind11_bindings.cpp:
        133-163; cuszp_wrapper.cpp:683-868).  All groups are encoded by one
        kernel launch."""
        batch = len(input_tensors)
        prefix_count, source_layers = int(prefix_count), int(source_layers)
        elements_per_layer = int(elements_per_layer)
        if (batch == 0 or len(compressed_buffers) != batch
                or (eps_overrides and len(eps_overrides) != batch)
                or len(layer_indices) == 0 or len(layer_indices) != len(group_sizes)
                or prefix_count <= 0 or source_layers <= 0 or elements_per_layer <= 0
                or not self._fixed_1d_float()):
            return False, [], []
        if any(int(g) <= 0 for g in group_sizes) or sum(int(g) for g in group_sizes) != batch:
            return False, [], []
        if not all(self._check_layer_index(i, source_layers) for i in layer_indices):
            return False, [], []
        source_elements = prefix_count * source_layers * elements_per_layer
        capacities = []
        unit = 0
        for idx, g in zip(layer_indices, group_sizes):
            required = _lib.ckv_estimate_compressed_buffer_size(
                prefix_count * idx.numel() * elements_per_layer * 4)
            for _ in range(int(g)):
                t, o = input_tensors[unit], compressed_buffers[unit]
                if (not self._on_device(t) or not self._on_device(o)
                        or t.dtype != torch.bfloat16 or o.dtype != torch.uint8
                        or not t.is_contiguous() or not o.is_contiguous()
                        or t.numel() < source_elements or o.numel() < required):
                    return False, [], []
                capacities.append(o.numel())
                unit += 1
        sizes = (_ckv.c_size * batch)()
        bounds = (_ckv.c_float * batch)()
        ok = self._call(
            _lib.ckv_compress_batch_fixed_bf16_indexed_groups,
            _ckv.ptr_array([t.data_ptr() for t in input_tensors]),
            _ckv.ptr_array([o.data_ptr() for o in compressed_buffers]),
            _ckv.ptr_array([i.data_ptr() for i in layer_indices]),
            _ckv.size_array([i.numel() for i in layer_indices]),
            _ckv.size_array([int(g) for g in group_sizes]), len(group_sizes),
            prefix_count, source_layers, elements_per_layer,
            self._eps_list(eps_overrides, batch), batch, _ckv.size_array(capacities),
            sizes, bounds, _stream(self._device))
        if not ok:
            return False, [], []
        return True, [int(s) for s in sizes], [float(b) for b in bounds]

    # -- decompression ---------------------------------------------------
    def decompress(self, compressed_buffer, compressed_size, output_tensor,
                   actual_error_bound):
        """decompress (pybind11_bindings.cpp:164-173; cuszp_wrapper.cpp:870-943):
        FP32 output, asynchronous on the current stream."""
        if not compressed_buffer.is_cuda or not output_tensor.is_cuda:
            _report("Both compressed buffer and output tensor must be on GPU")
            return False
        if output_tensor.dtype != torch.float32 or not output_tensor.is_contiguous():
            _report("decompress expects a contiguous float32 output tensor")
            return False
        return self._call(_lib.ckv_decompress, compressed_buffer.data_ptr(),
                          int(compressed_size), output_tensor.data_ptr(),
                          output_tensor.numel(), float(actual_error_bound),
                          _stream(output_tensor.device))

    def decompress_batch(self, compressed_buffers, compressed_sizes, output_tensors,
                         actual_error_bounds):
        """decompress_batch (pybind11_bindings.cpp:174-189;
        cuszp_wrapper.cpp:944-1033): FP32 outputs, one launch."""
        batch = len(compressed_buffers)
        if batch == 0:
            return True
        if len(compressed_sizes) != batch or len(output_tensors) != batch \
                or len(actual_error_bounds) != batch:
            _report("cuSZp batch metadata lengths differ")
            return False
        for b, o, s in zip(compressed_buffers, output_tensors, compressed_sizes):
            if (not b.is_cuda or not o.is_cuda or o.dtype != torch.float32
                    or not o.is_contiguous() or int(s) == 0):
                _report("invalid tensor in cuSZp batch")
                return False
        return self._call(_lib.ckv_decompress_batch,
                          _ckv.ptr_array([b.data_ptr() for b in compressed_buffers]),
                          _ckv.size_array([int(s) for s in compressed_sizes]),
                          _ckv.ptr_array([o.data_ptr() for o in output_tensors]),
                          _ckv.size_array([o.numel() for o in output_tensors]),
                          _ckv.float_array([float(e) for e in actual_error_bounds]),
                          batch, _stream(output_tensors[0].device))

    def decompress_batch_fixed_bf16(self, compressed_buffers, compressed_sizes,
                                    output_tensor, num_elements_per_page,
                                    actual_error_bounds):
        """decompress_batch_fixed_bf16 (pybind11_bindings.cpp:190-207;
        cuszp_wrapper.cpp:1034-1110)."""
        batch = len(compressed_buffers)
        if batch == 0:
            return True
        n = int(num_elements_per_page)
        if (len(compressed_sizes) != batch or len(actual_error_bounds) != batch or n == 0
                or not output_tensor.is_cuda or output_tensor.dtype != torch.bfloat16
                or output_tensor.numel() < batch * n):
            _report("invalid cuSZp fixed BF16 batch metadata")
            return False
        if not self._fixed_1d_float():
            _report("BF16 batch kernel requires fixed 1D f32 cuSZp")
            return False
        for b, s in zip(compressed_buffers, compressed_sizes):
            if not b.is_cuda or int(s) == 0:
                _report("invalid compressed page in BF16 batch")
                return False
        return self._call(_lib.ckv_decompress_batch_fixed_bf16,
                          _ckv.ptr_array([b.data_ptr() for b in compressed_buffers]),
                          _ckv.size_array([int(s) for s in compressed_sizes]), batch,
                          output_tensor.data_ptr(), output_tensor.numel(), n,
                          _ckv.float_array([float(e) for e in actual_error_bounds]),
                          _stream(output_tensor.device))

    def decompress_batch_fixed_bf16_scatter(self, compressed_buffers, compressed_sizes,
                                            output_tensors, num_elements_per_page,
                                            destinations_per_page, elements_per_destination,
                                            actual_error_bounds):
        """decompress_batch_fixed_bf16_scatter (pybind11_bindings.cpp:208-230;
        cuszp_wrapper.cpp:1111-1212)."""
        batch = len(compressed_buffers)
        if batch == 0:
            return True
        per, epd = int(destinations_per_page), int(elements_per_destination)
        n = int(num_elements_per_page)
        if (len(compressed_sizes) != batch or len(actual_error_bounds) != batch or per == 0
                or epd == 0 or n != per * epd or len(output_tensors) != batch * per):
            _report("invalid cuSZp direct-scatter metadata")
            return False
        if not self._fixed_1d_float():
            _report("direct scatter requires fixed 1D f32 cuSZp")
            return False
        for b, s in zip(compressed_buffers, compressed_sizes):
            if not b.is_cuda or int(s) == 0:
                _report("invalid compressed direct-scatter page")
                return False
        for o in output_tensors:
            if (not o.is_cuda or o.dtype != torch.bfloat16 or not o.is_contiguous()
                    or o.numel() < epd):
                _report("invalid BF16 direct-scatter destination")
                return False
        return self._call(_lib.ckv_decompress_batch_fixed_bf16_scatter,
                          _ckv.ptr_array([b.data_ptr() for b in compressed_buffers]),
                          _ckv.size_array([int(s) for s in compressed_sizes]), batch,
                          _ckv.ptr_array([o.data_ptr() for o in output_tensors]),
                          len(output_tensors), n, per, epd,
                          _ckv.float_array([float(e) for e in actual_error_bounds]),
                          _stream(output_tensors[0].device))

    def decompress_batch_fixed_bf16_indexed_scatter(self, compressed_buffers,
                                                    compressed_sizes, output_tensors,
                                                    layer_indices, prefix_count,
                                                    source_layers, elements_per_layer,
                                                    actual_error_bounds):
        """decompress_batch_fixed_bf16_indexed_scatter (pybind11_bindings.cpp:
        232-256; cuszp_wrapper.cpp:1214-1313)."""
        batch = len(compressed_buffers)
        if batch == 0:
            return True
        prefix_count, source_layers = int(prefix_count), int(source_layers)
        elements_per_layer = int(elements_per_layer)
        if (len(compressed_sizes) != batch or len(actual_error_bounds) != batch
                or len(output_tensors) != batch or prefix_count <= 0 or source_layers <= 0
                or elements_per_layer <= 0
                or not self._check_layer_index(layer_indices, source_layers)
                or not self._fixed_1d_float()):
            return False
        source_elements = prefix_count * source_layers * elements_per_layer
        for b, s, o in zip(compressed_buffers, compressed_sizes, output_tensors):
            if (not self._on_device(b) or int(s) == 0 or not self._on_device(o)
                    or o.dtype != torch.bfloat16 or not o.is_contiguous()
                    or o.numel() < source_elements):
                return False
        return self._call(_lib.ckv_decompress_batch_fixed_bf16_indexed_scatter,
                          _ckv.ptr_array([b.data_ptr() for b in compressed_buffers]),
                          _ckv.size_array([int(s) for s in compressed_sizes]), batch,
                          _ckv.ptr_array([o.data_ptr() for o in output_tensors]),
                          layer_indices.data_ptr(), layer_indices.numel(), prefix_count,
                          source_layers, elements_per_layer,
                          _ckv.float_array([float(e) for e in actual_error_bounds]),
                          _stream(self._device))

    # -- misc ----------------------------------------------------------------
    @staticmethod
    def estimate_compressed_buffer_size(original_size: int) -> int:
        """estimate_compressed_buffer_size (cuszp_wrapper.cpp:1319-1321)."""
        return int(_lib.ckv_estimate_compressed_buffer_size(int(original_size)))

    def get_config(self) -> CompressionConfig:
        return _copy_config(self._config)

    def update_config(self, config: CompressionConfig) -> None:
        self._config = _copy_config(config)
        _lib.ckv_update_config(self._ctx, self._config._as_c())

    # -- extensions ------------------------------------------------------------
    def set_zero_fill(self, zero_fill: bool) -> None:
        """Decode rate-0 blocks as zeros instead of leaving them untouched."""
        _lib.ckv_set_zero_fill(self._ctx, int(bool(zero_fill)))

    def device_status(self, reset: bool = True) -> int:
        """Status bits recorded by asynchronous decodes (waits for the stream)."""
        bits = _ckv.C.c_uint32(0)
        self._call(_lib.ckv_device_status, _stream(self._device), int(reset),
                   _ckv.C.byref(bits))
        return int(bits.value)


def kernel_launches() -> int:
    """Kernel launches issued by libckv in this process."""
    return int(_lib.ckv_kernel_launches())
