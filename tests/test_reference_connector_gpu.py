"""The drop-in check: the reference's own vLLM connector, unmodified, on libckv.

The reference connector (integration/compression_pipeline/
vllm_v1_compressed_offload.py) imports the module ``cuszp_wrapper_cpp`` by
name (:41-45) and drives every cuSZp call through it.  Here that name
resolves to this repository's ``cuszp_wrapper_cpp`` (ctypes over libckv)
instead of the reference's pybind11 extension, and the reference's own
connector tests (tests/test_vllm_v1_compressed_offload.py) run against it
unchanged.

The connector and its tests are the reference's files, byte-compiled where
they lie by oracle/build.py (stage_connector) into oracle/_ref/py, which
travels with the tree to the GPU box (the box has no reference checkout);
a finder on sys.meta_path loads them from there.
Out of scope: the upstream cuSZp ``plain`` and ``outlier`` encoders, which
this build does not implement (their ``compress`` returns False).  So the
``plain`` / ``outlier`` cases of test_real_cuszp_page_round_trip_through_
vllm_specs are not run, and the two tests that leave the connector at its
default mode, ``plain`` (:654 mixed layer policy, :830 async store), are
expected to fail as written; each also runs with only that default changed
to ``fixed`` (the handlers' ``cuszp_mode`` argument, nothing else).
"""
from __future__ import annotations

import importlib
import importlib.abc
import importlib.machinery
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "reducing-pcie-bottlenecks-for-llm-serving-with-cuszp-compressed-kv-cache-transfer_b200"
REF_PY = ROOT / "oracle" / "_ref" / "py"
REF_TESTS = REF_PY / "ref_tests" / "test_vllm_v1_compressed_offload.refpyc"
REF_PACKAGES = ("integration", "integration.compression_pipeline")

# (reference test function, its parameters); line numbers are the function's
# line in the reference's tests/test_vllm_v1_compressed_offload.py
CASES = [
    ("test_native_fixed_batch_compression_round_trip", {}),                     # :8
    ("test_native_fixed_bf16_indexed_batch_round_trip", {}),                    # :47
    ("test_adaptive_controller_uses_deadline_pressure_and_layer_caps", {}),     # :115
    ("test_restore_cost_model_finds_bandwidth_break_even", {}),                 # :154
    ("test_adaptive_cost_gate_falls_back_to_raw_when_restore_cannot_win", {}),  # :175
    ("test_joint_gate_selects_fastest_calibrated_cuszp_mode", {}),              # :199
    ("test_real_cuszp_page_round_trip_through_vllm_specs", {"cuszp_mode": "fixed"}),  # :233
    ("test_batched_restore_round_trip_for_multiple_pinned_pages", {}),          # :291
    ("test_fixed_bf16_batched_fast_path_round_trip", {"adaptive_uniform": False}),   # :343
    ("test_fixed_bf16_batched_fast_path_round_trip", {"adaptive_uniform": True}),
    ("test_adaptive_fixed_segments_use_cross_page_bf16_batch_path", {"lower_bound": 0.0}),  # :462
    ("test_adaptive_fixed_segments_use_cross_page_bf16_batch_path", {"lower_bound": 1e-4}),
    ("test_mixed_layer_policy_preserves_sensitive_layers_and_saves_bytes", {}),  # :654
    ("test_mixed_layer_policy_preserves_sensitive_layers_and_saves_bytes", {"mode": "fixed"}),
    ("test_int8_codec_reinterprets_uint8_backing_and_halves_bytes", {}),         # :719
    ("test_zero_bound_segment_skips_numeric_compressor_path", {}),               # :753
    ("test_cpu_lossless_codec_restores_page_and_counts_payload", {"codec": "zlib"}),  # :792
    ("test_cpu_lossless_codec_restores_page_and_counts_payload", {"codec": "zstd"}),
    ("test_cpu_lossless_codec_restores_page_and_counts_payload", {"codec": "lz4"}),
    ("test_async_store_waits_for_background_compression_and_restores_page", {}),  # :830
    ("test_async_store_waits_for_background_compression_and_restores_page", {"mode": "fixed"}),
    ("test_packed_store_aligns_raw_bf16_after_odd_compressed_payload", {}),      # :892
]

# tests that, as written, leave the handlers at their default mode, "plain"
PLAIN_DEFAULT = {
    "test_mixed_layer_policy_preserves_sensitive_layers_and_saves_bytes",
    "test_async_store_waits_for_background_compression_and_restores_page",
}

# reference tests that reach cuSZp (and so libckv) through the connector
CODEC_CASES = {
    "test_native_fixed_batch_compression_round_trip",
    "test_native_fixed_bf16_indexed_batch_round_trip",
    "test_real_cuszp_page_round_trip_through_vllm_specs",
    "test_fixed_bf16_batched_fast_path_round_trip",
    "test_adaptive_fixed_segments_use_cross_page_bf16_batch_path",
    "test_mixed_layer_policy_preserves_sensitive_layers_and_saves_bytes",
    "test_async_store_waits_for_background_compression_and_restores_page",
}


class _PackageLoader(importlib.abc.Loader):
    """The reference's package directories (no code of their own)."""

    def create_module(self, spec):
        return None

    def exec_module(self, module):
        pass


class _StagedFinder(importlib.abc.MetaPathFinder):
    """Finds the reference's staged, byte-compiled connector modules."""

    def find_spec(self, name, path=None, target=None):
        rel = name.replace(".", "/")
        if name in REF_PACKAGES:
            spec = importlib.util.spec_from_loader(name, _PackageLoader(), is_package=True)
            spec.submodule_search_locations = [str(REF_PY / rel)]
            return spec
        if name.startswith("integration."):
            f = REF_PY / (rel + ".refpyc")
            if f.exists():
                return importlib.util.spec_from_loader(
                    name, importlib.machinery.SourcelessFileLoader(name, str(f)))
        return None


def _staged():
    if not REF_TESTS.exists():
        pytest.skip("reference connector not staged in oracle/_ref/py "
                    "(run oracle/build.py where a reference checkout exists)")
    if str(PKG) in sys.path:   # this package first: its cuszp_wrapper_cpp
        sys.path.remove(str(PKG))
    sys.path.insert(0, str(PKG))
    if not any(isinstance(f, _StagedFinder) for f in sys.meta_path):
        sys.meta_path.insert(0, _StagedFinder())


def _reference_tests():
    _staged()
    name = "reference_connector_tests"
    if name in sys.modules:
        return sys.modules[name]
    loader = importlib.machinery.SourcelessFileLoader(name, str(REF_TESTS))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def test_reference_connector_binds_this_wrapper():
    """CPU: the unmodified connector imports and its cuszp_wrapper_cpp is this
    repository's module (ctypes over libckv), with the enum values the
    connector maps its mode names to."""
    _staged()
    import cuszp_wrapper_cpp as ours

    offload = importlib.import_module("integration.compression_pipeline.vllm_v1_compressed_offload")
    assert offload.cuszp_wrapper_cpp is ours
    assert Path(ours.__file__).resolve().parent == PKG.resolve()
    assert offload.CUSZP_MODES["fixed"] == ours.CuszpMode.MODE_FIXED
    assert Path(offload.__file__).suffix == ".refpyc"


def _case(name, kwargs):
    marks = []
    if name in PLAIN_DEFAULT and kwargs.get("mode") != "fixed":
        marks.append(pytest.mark.xfail(
            strict=True, reason="the connector's default cuszp_mode is 'plain', an upstream cuSZp "
                                "encoder this build does not implement"))
    return pytest.param(name, kwargs, marks=marks,
                        id=name + "".join(f"[{v}]" for v in kwargs.values()))


@pytest.mark.gpu
@pytest.mark.parametrize("name,kwargs", [_case(n, k) for n, k in CASES])
def test_reference_connector_test_passes_on_libckv(name, kwargs):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    mod = _reference_tests()
    import cuszp_wrapper_cpp as ours

    kwargs = dict(kwargs)
    mode = kwargs.pop("mode", None)
    offload = importlib.import_module("integration.compression_pipeline.vllm_v1_compressed_offload")
    handlers = offload.CompressedCpuGpuOffloadingHandlers
    init = handlers.__init__
    if mode is not None:
        def with_mode(self, *a, **kw):
            kw.setdefault("cuszp_mode", mode)
            init(self, *a, **kw)
        handlers.__init__ = with_mode
    try:
        before = ours.kernel_launches()
        getattr(mod, name)(**kwargs)
        torch.cuda.synchronize()
    finally:
        handlers.__init__ = init
    if name in CODEC_CASES:
        assert ours.kernel_launches() > before, "the connector did not reach libckv"
