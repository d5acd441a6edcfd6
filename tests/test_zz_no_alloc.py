"""The allocation-free compressor against the regular one (GPU).

ckv_compress_batch_fixed_bf16_noalloc serves callers that cannot allocate
device memory when they compress (an engine that reserved all free HBM for
its KV cache, or code that must avoid the synchronisation of cudaFree); its
scratch is a fixed device array inside libckv.  Called through the C ABI,
twice in a row on the same pages, it must give exactly the sizes, resolved
bounds and compressed bytes of ckv_compress_batch_fixed_bf16.  This file is
named to run after every other test file.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _pages(count, n, seed):
    g = torch.Generator().manual_seed(seed)
    scale = torch.empty(128).log_normal_(0.0, 0.5, generator=g)
    x = torch.randn(count, n, generator=g) * scale.repeat(n // 128 + 1)[:n]
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("count,n,eb", [(16, 229376, 1e-5), (5, 40001, 1e-4)])
def test_noalloc_matches_regular_entry_point(count, n, eb):
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv

    lib = _ckv.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pages = _pages(count, n, seed=n).to(dev)
    cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
    stream = torch.cuda.current_stream(dev).cuda_stream
    inputs = _ckv.ptr_array([pages[i].data_ptr() for i in range(count)])
    eps = _ckv.float_array([eb] * count)

    # the regular entry point, through a context
    ref_out = torch.full((count, cap), 0xCD, dtype=torch.uint8, device=dev)
    ctx = C.c_void_p()
    cfg = _ckv.Config(eb, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
    assert lib.ckv_create(cfg, 0, C.byref(ctx)) == 0
    ref_sizes = (C.c_size_t * count)()
    ref_bounds = (C.c_float * count)()
    assert lib.ckv_compress_batch_fixed_bf16(
        ctx, inputs, _ckv.ptr_array([ref_out[i].data_ptr() for i in range(count)]), eps,
        count, n, cap, ref_sizes, ref_bounds, stream) == 0
    lib.ckv_destroy(ctx)

    for call in range(2):
        out = torch.full((count, cap), 0xEF, dtype=torch.uint8, device=dev)
        sizes = (C.c_size_t * count)()
        bounds = (C.c_float * count)()
        status = lib.ckv_compress_batch_fixed_bf16_noalloc(
            inputs, _ckv.ptr_array([out[i].data_ptr() for i in range(count)]), eps, count, n,
            cap, eb, 1, sizes, bounds, stream)
        assert status == 0, f"call {call}: status {status}"
        assert list(sizes) == list(ref_sizes), f"call {call}"
        assert [C.c_float(b).value for b in bounds] == [C.c_float(b).value for b in ref_bounds]
        for i in range(count):
            s = sizes[i]
            assert torch.equal(out[i, :s], ref_out[i, :s]), f"call {call}, page {i}"


@pytest.mark.parametrize("n", [229376, 327680])   # both encoder slice geometries
def test_noalloc_allocates_no_device_memory_after_setup(n):
    """After the set-up call (batch 0), compress calls leave the driver's free
    device memory unchanged: torch.cuda.mem_get_info reads cudaMemGetInfo,
    which sees allocations that torch's caching allocator would hide."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv

    lib = _ckv.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    count, eb = 8, 1e-5
    pages = _pages(count, n, seed=7).to(dev)
    cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
    out = torch.empty((count, cap), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    inputs = _ckv.ptr_array([pages[i].data_ptr() for i in range(count)])
    outputs = _ckv.ptr_array([out[i].data_ptr() for i in range(count)])
    sizes = (C.c_size_t * count)()
    bounds = (C.c_float * count)()
    torch.cuda.synchronize(dev)

    assert lib.ckv_compress_batch_fixed_bf16_noalloc(
        None, None, None, 0, 0, 0, 0.0, 0, None, None, stream) == 0
    torch.cuda.synchronize(dev)
    free_before, _ = torch.cuda.mem_get_info(dev)
    for call in range(3):
        status = lib.ckv_compress_batch_fixed_bf16_noalloc(
            inputs, outputs, None, count, n, cap, eb, 1, sizes, bounds, stream)
        assert status == 0, f"call {call}: status {status}"
    torch.cuda.synchronize(dev)
    free_after, _ = torch.cuda.mem_get_info(dev)
    assert free_after == free_before, f"{free_before - free_after} bytes of device memory taken"


def test_noalloc_rejects_batches_above_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv

    lib = _ckv.load()
    dev = torch.device("cuda", 0)
    too_many = 4097  # CKV_NOALLOC_MAX_UNITS + 1
    page = torch.zeros(64, dtype=torch.bfloat16, device=dev)
    out = torch.empty(8 * 64 * 4, dtype=torch.uint8, device=dev)
    sizes = (C.c_size_t * too_many)()
    bounds = (C.c_float * too_many)()
    status = lib.ckv_compress_batch_fixed_bf16_noalloc(
        _ckv.ptr_array([page.data_ptr()] * too_many), _ckv.ptr_array([out.data_ptr()] * too_many),
        None, too_many, 64, out.numel(), 1e-4, 1, sizes, bounds,
        torch.cuda.current_stream(dev).cuda_stream)
    assert status == 1  # CKV_ERR_ARGUMENT, before any GPU work
