"""Store / restore pipeline (ckv_pipe_*) against the plain batched calls (GPU).

The pipeline must produce, page for page, the compressed bytes, sizes and
bounds of ckv_compress_batch_fixed_bf16 and restore exactly what
ckv_decompress_batch_fixed_bf16_scatter restores, for any chunking, while a
store and a restore run together on alternating host buffers.
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


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv

    lib = _ckv.load()
    ctx = C.c_void_p()
    cfg = _ckv.Config(1e-5, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
    assert lib.ckv_create(cfg, 0, C.byref(ctx)) == 0
    yield _ckv, lib, ctx
    lib.ckv_destroy(ctx)


def _reference(_ckv, lib, ctx, pages):
    count, n = pages.shape
    cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
    outs = torch.zeros(count, cap, dtype=torch.uint8, device="cuda")
    sizes = (C.c_size_t * count)()
    bounds = (C.c_float * count)()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ckv_compress_batch_fixed_bf16(
        ctx, _ckv.ptr_array([pages[i].data_ptr() for i in range(count)]),
        _ckv.ptr_array([outs[i].data_ptr() for i in range(count)]), None, count, n, cap, sizes,
        bounds, s) == 0
    restored = torch.empty_like(pages)
    assert lib.ckv_decompress_batch_fixed_bf16_scatter(
        ctx, _ckv.ptr_array([outs[i].data_ptr() for i in range(count)]), sizes, count,
        _ckv.ptr_array([restored[i].data_ptr() for i in range(count)]), count, n, 1, n, bounds,
        s) == 0
    torch.cuda.synchronize()
    return outs, list(sizes), [C.c_float(b).value for b in bounds], restored


@pytest.mark.parametrize("count,n,chunk", [(37, 229376, 8), (5, 40001, 2), (64, 36864, 64),
                                           (3, 1000, 7)])
def test_pipe_matches_plain_calls(env, count, n, chunk):
    _ckv, lib, ctx = env
    pages = _pages(count, n, seed=count * 7 + n).cuda()
    ref_outs, ref_sizes, ref_bounds, ref_restored = _reference(_ckv, lib, ctx, pages)

    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, chunk, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity(count, n))
        host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        sizes = (C.c_size_t * count)()
        bounds = (C.c_float * count)()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        s = torch.cuda.current_stream().cuda_stream
        ptrs = _ckv.ptr_array([pages[i].data_ptr() for i in range(count)])
        assert lib.ckv_pipe_store_bf16(pipe, ptrs, None, count, n, host.data_ptr(), cap, offsets,
                                       sizes, bounds, C.byref(total), 0, C.byref(ticket), s) == 0
        assert lib.ckv_pipe_wait(pipe, ticket.value) == 0
        assert lib.ckv_pipe_done(pipe, ticket.value) == 1
        assert list(sizes) == ref_sizes
        assert [C.c_float(b).value for b in bounds] == ref_bounds
        for i in range(count):
            assert offsets[i] % 16 == 0
            got = host[offsets[i]:offsets[i] + sizes[i]]
            assert torch.equal(got, ref_outs[i, :sizes[i]].cpu()), f"page {i}"
        restored = torch.full_like(pages, 7.0)
        t2 = C.c_uint64(0)
        assert lib.ckv_pipe_restore_bf16(
            pipe, host.data_ptr(), offsets, sizes, bounds, count, n,
            _ckv.ptr_array([restored[i].data_ptr() for i in range(count)]), ticket.value,
            C.byref(t2), s) == 0
        torch.cuda.synchronize()
        assert torch.equal(restored.view(torch.int16), ref_restored.view(torch.int16))
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_pipe_overlapped_store_and_restore(env):
    """Step k stores into slab k % 2 while step k-1's slab is restored."""
    _ckv, lib, ctx = env
    count, n = 40, 65536
    batches = [_pages(count, n, seed=100 + k).cuda() for k in range(4)]
    refs = [_reference(_ckv, lib, ctx, b)[3] for b in batches]
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 16, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity(count, n))
        slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * count)(), "s": (C.c_size_t * count)(),
                 "b": (C.c_float * count)(), "t": C.c_size_t(0)} for _ in range(2)]
        s = torch.cuda.current_stream().cuda_stream
        t_store = t_rest = 0
        outs = []
        for k in range(len(batches) + 1):
            ts = C.c_uint64(0)
            if k < len(batches):
                a = meta[k % 2]
                ptrs = _ckv.ptr_array([batches[k][i].data_ptr() for i in range(count)])
                assert lib.ckv_pipe_store_bf16(pipe, ptrs, None, count, n,
                                               slabs[k % 2].data_ptr(), cap, a["o"], a["s"],
                                               a["b"], C.byref(a["t"]), t_rest, C.byref(ts),
                                               s) == 0
            if k > 0:
                b = meta[(k + 1) % 2]
                out = torch.empty(count, n, dtype=torch.bfloat16, device="cuda")
                tr = C.c_uint64(0)
                assert lib.ckv_pipe_restore_bf16(
                    pipe, slabs[(k + 1) % 2].data_ptr(), b["o"], b["s"], b["b"], count, n,
                    _ckv.ptr_array([out[i].data_ptr() for i in range(count)]), t_store,
                    C.byref(tr), s) == 0
                t_rest = tr.value
                outs.append(out)
            t_store = ts.value
        torch.cuda.synchronize()
        for k, out in enumerate(outs):
            assert torch.equal(out.view(torch.int16), refs[k].view(torch.int16)), f"batch {k}"
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_pipe_back_to_back_single_chunk_jobs(env):
    """Jobs of one chunk each, stored on one stream and restored on another
    with no host synchronisation between them: consecutive jobs alternate
    the pipeline's staging and landing buffers, so job k+1 compresses while
    job k is still being copied out.  Every stored byte and every restored
    page matches the plain calls."""
    _ckv, lib, ctx = env
    count, n, jobs = 24, 65536, 8
    batches = [_pages(count, n, seed=300 + k).cuda() for k in range(4)]
    refs = [_reference(_ckv, lib, ctx, b) for b in batches]
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, count, C.byref(pipe)) == 0
    side = torch.cuda.Stream()
    try:
        cap = int(lib.ckv_pipe_host_capacity(count, n))
        slabs = [torch.zeros(cap, dtype=torch.uint8, pin_memory=True) for _ in range(jobs)]
        meta = [{"o": (C.c_size_t * count)(), "s": (C.c_size_t * count)(),
                 "b": (C.c_float * count)(), "t": C.c_size_t(0)} for _ in range(jobs)]
        outs = [torch.empty(count, n, dtype=torch.bfloat16, device="cuda") for _ in range(jobs)]
        main = torch.cuda.current_stream().cuda_stream
        stored = [0] * jobs
        for k in range(jobs + 1):
            if k < jobs:
                m = meta[k]
                b = batches[k % len(batches)]
                ts = C.c_uint64(0)
                assert lib.ckv_pipe_store_bf16(
                    pipe, _ckv.ptr_array([b[i].data_ptr() for i in range(count)]), None, count, n,
                    slabs[k].data_ptr(), cap, m["o"], m["s"], m["b"], C.byref(m["t"]), 0,
                    C.byref(ts), main) == 0
                stored[k] = ts.value
            if k >= 1:   # restore job k-1 on the side stream, after its store
                r = k - 1
                m = meta[r]
                tr = C.c_uint64(0)
                assert lib.ckv_pipe_restore_bf16(
                    pipe, slabs[r].data_ptr(), m["o"], m["s"], m["b"], count, n,
                    _ckv.ptr_array([outs[r][i].data_ptr() for i in range(count)]), stored[r],
                    C.byref(tr), side.cuda_stream) == 0
        torch.cuda.synchronize()
        for r in range(jobs):
            ref_outs, ref_sizes, ref_bounds, ref_restored = refs[r % len(batches)]
            assert list(meta[r]["s"]) == ref_sizes, f"job {r}"
            assert torch.equal(outs[r].view(torch.int16), ref_restored.view(torch.int16)), f"job {r}"
            host = ref_outs.cpu()
            for i in range(count):
                o, sz = meta[r]["o"][i], ref_sizes[i]
                assert torch.equal(slabs[r][o:o + sz], host[i, :sz]), f"job {r} page {i}"
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_pipe_rejects_small_host_buffer(env):
    _ckv, lib, ctx = env
    count, n = 4, 32768
    pages = _pages(count, n, seed=5).cuda()
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 2, C.byref(pipe)) == 0
    try:
        host = torch.empty(1024, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        sizes = (C.c_size_t * count)()
        bounds = (C.c_float * count)()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        st = lib.ckv_pipe_store_bf16(
            pipe, _ckv.ptr_array([pages[i].data_ptr() for i in range(count)]), None, count, n,
            host.data_ptr(), host.numel(), offsets, sizes, bounds, C.byref(total), 0,
            C.byref(ticket), torch.cuda.current_stream().cuda_stream)
        assert st == 4  # CKV_ERR_CAPACITY
        torch.cuda.synchronize()
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_pipe_layer_groups_match_plain_calls(env):
    """The C3 layout: pages of 28 layers, 21 at 1e-4 and 7 at 1e-5 (the
    reference's calibrated profile), stored as two segments per page through
    the pipeline; bytes and bounds equal compress_batch_fixed_bf16_indexed_groups,
    the restore equals decompress_batch_fixed_bf16_indexed_scatter per group."""
    import cuszp_wrapper_cpp as cpp

    _ckv, lib, ctx = env
    layers, prefix, epl, count, chunk = 28, 2, 4096, 9, 4
    low = [0, 1, 2, 5, 19, 20, 21]
    high = [i for i in range(layers) if i not in low]
    pages = _pages(count, prefix * layers * epl, seed=31).cuda()
    groups = [torch.tensor(high, device="cuda"), torch.tensor(low, device="cuda")]
    eps = [1e-4, 1e-5]

    cfg = cpp.CompressionConfig(error_bound=1e-5, use_relative_error=True,
                                processing_dim=cpp.CuszpDim.DIM_1D,
                                encoding_mode=cpp.CuszpMode.MODE_FIXED,
                                data_type=cpp.CuszpType.TYPE_FLOAT)
    w = cpp.CuSZpWrapper(cfg, 0)
    caps = [int(w.estimate_compressed_buffer_size(prefix * len(g) * epl * 4)) for g in (high, low)]
    outs = [torch.zeros(caps[0], dtype=torch.uint8, device="cuda") for _ in range(count)] + \
           [torch.zeros(caps[1], dtype=torch.uint8, device="cuda") for _ in range(count)]
    ok, ref_sizes, ref_bounds = w.compress_batch_fixed_bf16_indexed_groups(
        [pages[i] for i in range(count)] * 2, outs, groups, [count, count], prefix, layers, epl,
        [eps[0]] * count + [eps[1]] * count)
    assert ok
    ref_restored = torch.zeros_like(pages)
    dests = [ref_restored[i] for i in range(count)]
    assert w.decompress_batch_fixed_bf16_indexed_scatter(
        outs[:count], ref_sizes[:count], dests, groups[0], prefix, layers, epl, ref_bounds[:count])
    assert w.decompress_batch_fixed_bf16_indexed_scatter(
        outs[count:], ref_sizes[count:], dests, groups[1], prefix, layers, epl, ref_bounds[count:])
    torch.cuda.synchronize()

    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, chunk, C.byref(pipe)) == 0
    try:
        G = len(groups)
        sel = (C.c_size_t * G)(*[len(high), len(low)])
        idx = (C.c_void_p * G)(*[g.data_ptr() for g in groups])
        epsa = (C.c_float * G)(*eps)
        cap = int(lib.ckv_pipe_host_capacity_groups(count, sel, G, prefix, epl))
        host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * (count * G))()
        sizes = (C.c_size_t * (count * G))()
        bounds = (C.c_float * (count * G))()
        total = C.c_size_t(0)
        t1, t2 = C.c_uint64(0), C.c_uint64(0)
        s = torch.cuda.current_stream().cuda_stream
        ptrs = _ckv.ptr_array([pages[i].data_ptr() for i in range(count)])
        assert lib.ckv_pipe_store_bf16_groups(pipe, ptrs, count, idx, sel, G, prefix, layers, epl,
                                              epsa, host.data_ptr(), cap, offsets, sizes, bounds,
                                              C.byref(total), 0, C.byref(t1), s) == 0
        assert lib.ckv_pipe_wait(pipe, t1.value) == 0
        for i in range(count):
            for g in range(G):
                j, r = i * G + g, g * count + i
                assert sizes[j] == ref_sizes[r]
                assert C.c_float(bounds[j]).value == C.c_float(ref_bounds[r]).value
                got = host[offsets[j]:offsets[j] + sizes[j]]
                assert torch.equal(got, outs[r][:sizes[j]].cpu()), (i, g)
        restored = torch.zeros_like(pages)
        assert lib.ckv_pipe_restore_bf16_groups(
            pipe, host.data_ptr(), offsets, sizes, bounds, count, idx, sel, G, prefix, layers, epl,
            _ckv.ptr_array([restored[i].data_ptr() for i in range(count)]), t1.value,
            C.byref(t2), s) == 0
        torch.cuda.synchronize()
        assert torch.equal(restored.view(torch.int16), ref_restored.view(torch.int16))
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_pipe_tickets_retire(env):
    """A ticket older than the pipeline's 64 ticket events reads as complete
    (done 1, wait and join return at once) instead of aliasing newer work."""
    _ckv, lib, ctx = env
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 8, C.byref(pipe)) == 0
    try:
        s = torch.cuda.current_stream().cuda_stream
        first, t = C.c_uint64(0), C.c_uint64(0)
        assert lib.ckv_pipe_record(pipe, s, C.byref(first)) == 0
        for _ in range(64):
            assert lib.ckv_pipe_record(pipe, s, C.byref(t)) == 0
        assert t.value == first.value + 64
        assert lib.ckv_pipe_done(pipe, first.value) == 1
        assert lib.ckv_pipe_wait(pipe, first.value) == 0
        assert lib.ckv_pipe_join(pipe, first.value, s) == 0
        assert lib.ckv_pipe_done(pipe, t.value + 1) == -1
        assert lib.ckv_pipe_wait(pipe, t.value) == 0
        assert lib.ckv_pipe_done(pipe, t.value) == 1
    finally:
        lib.ckv_pipe_destroy(pipe)
