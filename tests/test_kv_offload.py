"""The offload job layer (kv_offload.py): on-host job format and page store on
CPU; store / load jobs through the handlers against the plain calls on GPU."""
import ctypes as C

import numpy as np
import pytest
import torch

import kv_offload as ko


# ---------------------------------------------------------------- CPU


def test_job_header_round_trip():
    count, n = 5, 229376
    offsets = (C.c_size_t * count)(0, 320, 704, 1024, 4096)
    sizes = (C.c_size_t * count)(300, 384, 300, 3000, 16)
    bounds = (C.c_float * count)(1e-4, 2e-4, 3e-4, 4e-4, 5e-4)
    hdr = ko.JobHeader.bytes_for(count)
    assert hdr % 256 == 0
    slab = torch.zeros(hdr + 4112, dtype=torch.uint8)
    ko.JobHeader.write(slab, n, 1e-5, True, offsets, sizes, bounds, 4112)
    job = ko.JobHeader.read(slab)
    assert job["count"] == count and job["n"] == n and job["relative"]
    assert job["payload_at"] == hdr and job["payload_bytes"] == 4112
    assert np.float32(job["eps"]) == np.float32(1e-5)
    assert job["offsets"].tolist() == list(offsets)
    assert job["sizes"].tolist() == list(sizes)
    assert job["bounds"].tolist() == [np.float32(b) for b in bounds]


def test_job_header_rejects_bad_slabs():
    count = 2
    offsets = (C.c_size_t * count)(0, 64)
    sizes = (C.c_size_t * count)(64, 64)
    bounds = (C.c_float * count)(1.0, 1.0)
    hdr = ko.JobHeader.bytes_for(count)
    slab = torch.zeros(hdr + 128, dtype=torch.uint8)
    ko.JobHeader.write(slab, 1000, 1e-4, False, offsets, sizes, bounds, 128)
    ko.JobHeader.read(slab)
    bad = slab.clone()
    bad[0] = ord("X")
    with pytest.raises(ValueError):
        ko.JobHeader.read(bad)
    with pytest.raises(ValueError):
        ko.JobHeader.read(slab[: hdr + 64])          # payload cut short
    big = (C.c_size_t * count)(64, 200)
    ko.JobHeader.write(slab, 1000, 1e-4, False, offsets, big, bounds, 128)
    with pytest.raises(ValueError):
        ko.JobHeader.read(slab)                       # page past the payload


def test_job_header_layer_groups_round_trip():
    count, layers, prefix = 3, 28, 2
    low = (0, 1, 2, 5, 19, 20, 21)
    high = tuple(i for i in range(layers) if i not in low)
    groups = [(1e-5, low), (1e-4, high)]
    offsets = (C.c_size_t * (2 * count))(0, 512, 4096, 4608, 8192, 8704)
    sizes = (C.c_size_t * (2 * count))(500, 3000, 500, 3000, 500, 3000)
    bounds = (C.c_float * (2 * count))(1e-5, 1e-4, 2e-5, 2e-4, 3e-5, 3e-4)
    hdr = ko.JobHeader.bytes_for(count, 2, layers)
    assert hdr % 256 == 0
    slab = torch.zeros(hdr + 11704, dtype=torch.uint8)
    ko.JobHeader.write(slab, prefix * layers * 4096, 1e-4, True, offsets, sizes, bounds, 11704,
                       groups, prefix, layers)
    job = ko.JobHeader.read(slab)
    assert job["count"] == count and job["segments"] == 2 and job["payload_at"] == hdr
    assert job["prefix"] == prefix and job["layers"] == layers
    assert [sel for _b, sel in job["groups"]] == [low, high]
    assert [np.float32(b) for b, _s in job["groups"]] == [np.float32(1e-5), np.float32(1e-4)]
    assert job["sizes"].tolist() == list(sizes)
    assert job["bounds"].tolist() == [np.float32(b) for b in bounds]
    bad = slab.clone()
    bad[ko.JobHeader._HEAD.size + 3] = 7          # layer 3 in a segment that does not exist
    with pytest.raises(ValueError):
        ko.JobHeader.read(bad)


def test_job_header_raw_entries():
    """Raw entries are flagged in the page table and must hold exactly the
    segment's BF16 bytes."""
    count, n = 3, 36864
    offsets = (C.c_size_t * count)(0, 73728, 80000)
    sizes = (C.c_size_t * count)(2 * n, 5000, 2 * n)
    bounds = (C.c_float * count)(0.0, 1e-4, 0.0)
    hdr = ko.JobHeader.bytes_for(count)
    slab = torch.zeros(hdr + 160000, dtype=torch.uint8)
    ko.JobHeader.write(slab, n, 1e-4, True, offsets, sizes, bounds, 160000,
                       raw=[True, False, True])
    job = ko.JobHeader.read(slab)
    assert job["raw"].tolist() == [True, False, True] and job["coded"] == n
    ko.JobHeader.write(slab, 8192, 1e-4, True, offsets, sizes, bounds, 160000,
                       raw=[True, False, True], coded=36864)
    with pytest.raises(ValueError):
        ko.JobHeader.read(slab)                 # a raw entry of 2 * 36864 bytes for 8192 elements
    sizes[0] = sizes[2] = 2 * 8192
    ko.JobHeader.write(slab, 8192, 1e-4, True, offsets, sizes, bounds, 160000,
                       raw=[True, False, True], coded=36864)
    job = ko.JobHeader.read(slab)
    assert job["coded"] == 36864 and job["n"] == 8192


def test_job_header_codecs():
    count, n = 2, 8192
    offsets = (C.c_size_t * count)(0, 8208)
    sizes = (C.c_size_t * count)(n + 4, n + 4)
    bounds = (C.c_float * count)(0.0, 0.0)
    hdr = ko.JobHeader.bytes_for(count)
    slab = torch.zeros(hdr + 16416, dtype=torch.uint8)
    ko.JobHeader.write(slab, n, 1e-4, True, offsets, sizes, bounds, 16416, codec="int8")
    assert ko.JobHeader.read(slab)["codec"] == "int8"
    sizes[1] = n + 8
    ko.JobHeader.write(slab, n, 1e-4, True, offsets, sizes, bounds, 16416, codec="int8")
    with pytest.raises(ValueError):
        ko.JobHeader.read(slab)                 # an INT8 page is n + 4 bytes
    sizes[0] = sizes[1] = 2 * n
    offsets[1] = 2 * n
    slab = torch.zeros(hdr + 4 * n, dtype=torch.uint8)
    ko.JobHeader.write(slab, n, 1e-4, True, offsets, sizes, bounds, 4 * n, codec="raw")
    job = ko.JobHeader.read(slab)
    assert job["codec"] == "raw" and job["raw"].tolist() == [True, True]


def test_layer_bounds_group_like_the_reference():
    """Segments are the distinct bounds in ascending order, each with its
    layers in ascending order; missing layers take the handler's bound."""
    e = ko._Engine.__new__(ko._Engine)
    e.n, e.error_bound, e.device = 2 * 28 * 4096, 1e-4, "cpu"
    low = [0, 1, 2, 5, 19, 20, 21]
    e._set_groups({i: 1e-5 for i in low} | {i: 1e-4 for i in range(28) if i not in low}, 2)
    assert e.segments == 2 and e.epl == 4096 and e.layers == 28
    assert e.groups[0] == (1e-5, tuple(low))
    assert e.groups[1][1] == tuple(i for i in range(28) if i not in low)
    assert list(e.sel) == [7, 21] and e.segment_numel(0) == 2 * 7 * 4096
    e._set_groups([3e-4] * 28, 2)                 # one bound: whole pages
    assert e.groups is None and e.segments == 1 and e.error_bound == 3e-4
    e._set_groups([1e-4] * 27 + [0.0], 2)         # a zero bound: a raw segment, first
    assert e.groups[0] == (0.0, (27,)) and e.cg == [1] and list(e.sel) == [27]
    with pytest.raises(ValueError):
        e._set_groups([1e-4] * 27 + [1e-5], 2)    # a compressed segment below 36864 elements
    with pytest.raises(ValueError):
        e._set_groups([1e-4] * 27 + [1e-5], 3)    # page does not split


def test_page_store_overwrite_evict_and_recycle():
    store = ko.CompressedPageStore(allocate=lambda n: torch.empty(n, dtype=torch.uint8))
    buffers = []

    def slab_with(pages):
        sid = store._take_slab(1024, 256, lambda t: None)
        buffers.append(store.slab(sid).buffer)
        entries = []
        for k, cpu in enumerate(pages):
            rec = ko._PageRecord(sid, (64 * k,), (64,), (0.5,), 32)
            entries.append((cpu, rec, ko.CompressedBundle((), 64, 64)))
        store.put_many_packed(entries)
        return sid

    slab_with([1, 2, 3])
    assert len(store) == 3 and store.record(2).offsets == (64,)
    s2 = slab_with([3, 4])             # block 3 moves to the new slab
    assert store.record(3).slab == s2 and len(store) == 4
    store.evict([1, 2])                # the first slab is unreferenced now
    assert len(store._free) == 1 and store._free[0][0] is buffers[0]
    with pytest.raises(KeyError):
        store.get(1)
    s3 = slab_with([7])                # reuses the freed buffer
    assert store.slab(s3).buffer is buffers[0] and not store._free


def test_page_store_reserve_fills_the_pool_first():
    made = []

    def allocate(n):
        made.append(n)
        return torch.empty(n, dtype=torch.uint8)

    store = ko.CompressedPageStore(allocate=allocate)
    store.reserve(4096, 2)
    assert made == [4096, 4096] and len(store._free) == 2
    reserved = {id(b) for b, _t in store._free}
    a = store._take_slab(1000, 0, lambda t: None)
    b = store._take_slab(4096, 0, lambda t: None)
    assert {id(store.slab(a).buffer), id(store.slab(b).buffer)} == reserved
    assert made == [4096, 4096] and not store._free     # no allocation for the first jobs
    store._take_slab(64, 0, lambda t: None)
    assert made == [4096, 4096, 64]


# ---------------------------------------------------------------- GPU


def _kv(blocks, page_shape, seed):
    g = torch.Generator().manual_seed(seed)
    n = int(np.prod(page_shape))
    scale = torch.empty(page_shape[-1]).log_normal_(0.0, 0.5, generator=g)
    x = torch.randn(blocks, n, generator=g) * scale.repeat(n // page_shape[-1])
    return x.to(torch.bfloat16).view(blocks, *page_shape)


@pytest.mark.gpu
def test_handlers_store_then_load_match_plain_calls():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp as cpp

    shape = (2, 28, 2, 16, 128)
    kv = _kv(64, shape, seed=11).cuda()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-5, device_id=0, chunk_pages=16)
    try:
        gpu_ids = np.array([3, 9, 10, 11, 40, 63, 0, 5, 22, 31], dtype=np.int64)
        cpu_ids = np.arange(100, 100 + len(gpu_ids), dtype=np.int64)
        assert h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        done = h.gpu_to_cpu_handler.get_finished()
        assert [(r.job_id, r.success) for r in done] == [(1, True)]

        # the same pages through the plain wrapper calls
        cfg = cpp.CompressionConfig(error_bound=1e-5, use_relative_error=True,
                                    processing_dim=cpp.CuszpDim.DIM_1D,
                                    encoding_mode=cpp.CuszpMode.MODE_FIXED,
                                    data_type=cpp.CuszpType.TYPE_FLOAT)
        w = cpp.CuSZpWrapper(cfg, 0)
        n = kv[0].numel()
        pages = [kv[i].view(-1) for i in gpu_ids]
        outs = [torch.empty(w.estimate_compressed_buffer_size(n * 4), dtype=torch.uint8,
                            device="cuda") for _ in pages]
        ok, sizes, bounds = w.compress_batch_fixed_bf16(pages, outs, [1e-5] * len(pages))
        assert ok
        for k, cpu in enumerate(cpu_ids):
            seg = h.store.get(int(cpu)).segments[0]
            assert seg.compressed_size == sizes[k]
            assert np.float32(seg.actual_error_bound) == np.float32(bounds[k])
            assert torch.equal(seg.payload, outs[k][: sizes[k]].cpu())

        # load into other GPU blocks, in another order
        dst_gpu = np.array([50, 51, 52, 53, 54, 55, 56, 57, 58, 59], dtype=np.int64)
        order = np.array([9, 0, 1, 8, 2, 7, 3, 6, 4, 5])
        assert h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids[order], dst_gpu))
        h.cpu_to_gpu_handler.wait({2})
        assert [r.success for r in h.cpu_to_gpu_handler.get_finished()] == [True]
        restored = torch.zeros(len(pages) * n, dtype=torch.bfloat16, device="cuda")
        assert w.decompress_batch_fixed_bf16(outs, sizes, restored, n, bounds)
        torch.cuda.synchronize()
        ref = restored.view(len(pages), n)
        for j, k in enumerate(order):
            assert torch.equal(kv[dst_gpu[j]].view(-1).view(torch.int16), ref[k].view(torch.int16))

        # the job restored from its slab bytes alone
        slab = h.store.slab(h.store.record(int(cpu_ids[0])).slab).buffer
        dst = [torch.empty(n, dtype=torch.bfloat16, device="cuda") for _ in pages]
        t = ko.restore_job(slab, dst, h.engine)
        assert h.engine.lib.ckv_pipe_wait(h.engine.pipe, t) == 0
        for k in range(len(pages)):
            assert torch.equal(dst[k].view(torch.int16), ref[k].view(torch.int16))
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_overlapping_jobs_and_slab_reuse():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    shape = (2, 4, 2, 16, 128)
    kv = _kv(96, shape, seed=12).cuda()
    snapshot = kv.clone()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=8)
    try:
        # store blocks 0-31 as job 1, 32-63 as job 2; load job 1's pages into
        # 64-95 while job 2 is still being stored
        h.gpu_to_cpu_handler.transfer_async(1, (np.arange(0, 32), np.arange(1000, 1032)))
        h.gpu_to_cpu_handler.transfer_async(2, (np.arange(32, 64), np.arange(2000, 2032)))
        h.cpu_to_gpu_handler.transfer_async(3, (np.arange(1000, 1032), np.arange(64, 96)))
        h.gpu_to_cpu_handler.wait({1, 2})
        h.cpu_to_gpu_handler.wait({3})
        torch.cuda.synchronize()
        first = kv[64:96].clone()
        # overwrite job 1's CPU blocks (its slab returns to the pool) and
        # load them again: the decode must match the first load bit for bit
        h.store.evict(range(1000, 1032))
        h.gpu_to_cpu_handler.transfer_async(4, (np.arange(0, 32), np.arange(1000, 1032)))
        h.cpu_to_gpu_handler.transfer_async(5, (np.arange(1000, 1032), np.arange(64, 96)))
        h.cpu_to_gpu_handler.wait({5})
        torch.cuda.synchronize()
        assert torch.equal(kv[64:96].view(torch.int16), first.view(torch.int16))
        assert torch.equal(kv[:64].view(torch.int16), snapshot[:64].view(torch.int16))
        err = (kv[64:96].float() - snapshot[:32].float()).abs()
        assert bool((err <= 1e-4 * 2 * snapshot[:32].float().abs().amax() + 1e-7 +
                     snapshot[:32].float().abs() * 2 ** -8).all())
        got = {r.job_id for r in h.gpu_to_cpu_handler.get_finished()}
        got |= {r.job_id for r in h.cpu_to_gpu_handler.get_finished()}
        assert got == {1, 2, 3, 4, 5}
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_order_jobs_after_the_callers_stream():
    """Each direction issues on a stream of its own: a store must still see
    the blocks as the caller's stream last wrote them (here after a ~10 ms
    sleep kernel, so a store that did not wait would compress the old
    values), and the caller's current stream is left as it was."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    shape = (2, 4, 2, 16, 128)
    kv = _kv(64, shape, seed=13).cuda()
    new = _kv(32, shape, seed=14).cuda()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=8)
    try:
        caller = torch.cuda.current_stream()
        torch.cuda._sleep(20_000_000)
        kv[:32].copy_(new)
        h.gpu_to_cpu_handler.transfer_async(1, (np.arange(0, 32), np.arange(1000, 1032)))
        assert torch.cuda.current_stream() == caller
        h.cpu_to_gpu_handler.transfer_async(2, (np.arange(1000, 1032), np.arange(32, 64)))
        assert torch.cuda.current_stream() == caller
        h.gpu_to_cpu_handler.wait({1})
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        first = kv[32:64].clone()
        x = new.float()
        err = (first.float() - x).abs()
        assert bool((err <= 1e-4 * 2 * x.abs().amax() + 1e-7 + x.abs() * 2 ** -8).all())
        # the same blocks stored and loaded again with nothing pending on the
        # caller's stream: bit for bit the same restore
        h.gpu_to_cpu_handler.transfer_async(3, (np.arange(0, 32), np.arange(3000, 3032)))
        h.cpu_to_gpu_handler.transfer_async(4, (np.arange(3000, 3032), np.arange(32, 64)))
        h.cpu_to_gpu_handler.wait({4})
        torch.cuda.synchronize()
        assert torch.equal(kv[32:64].view(torch.int16), first.view(torch.int16))
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_layer_groups_match_plain_calls():
    """The mixed per-layer profile (7 layers at 1e-5, 21 at 1e-4) through the
    handlers: two segments per page equal compress_batch_fixed_bf16_indexed
    per group; a load restores what decompress_batch_fixed_bf16_indexed_scatter
    restores, and so does the job read back from its slab bytes."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp as cpp

    shape = (2, 28, 2, 16, 128)
    layers, prefix, epl = 28, 2, 2 * 16 * 128
    low = [0, 1, 2, 5, 19, 20, 21]
    high = [i for i in range(layers) if i not in low]
    bounds_of = {i: (1e-5 if i in low else 1e-4) for i in range(layers)}
    kv = _kv(24, shape, seed=13).cuda()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=4,
                                              layer_bounds=bounds_of)
    try:
        gpu_ids = np.array([1, 4, 7, 8, 9, 15, 16, 23, 0], dtype=np.int64)
        cpu_ids = np.arange(300, 300 + len(gpu_ids), dtype=np.int64)
        assert h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        assert [r.success for r in h.gpu_to_cpu_handler.get_finished()] == [True]

        cfg = cpp.CompressionConfig(error_bound=1e-4, use_relative_error=True,
                                    processing_dim=cpp.CuszpDim.DIM_1D,
                                    encoding_mode=cpp.CuszpMode.MODE_FIXED,
                                    data_type=cpp.CuszpType.TYPE_FLOAT)
        w = cpp.CuSZpWrapper(cfg, 0)
        pages = [kv[i].view(-1) for i in gpu_ids]
        ref = {}
        for g, (eb, sel) in enumerate([(1e-5, low), (1e-4, high)]):
            index = torch.tensor(sel, device="cuda")
            outs = [torch.empty(w.estimate_compressed_buffer_size(prefix * len(sel) * epl * 4),
                                dtype=torch.uint8, device="cuda") for _ in pages]
            ok, sizes, bounds = w.compress_batch_fixed_bf16_indexed(
                pages, outs, index, prefix, layers, epl, [eb] * len(pages))
            assert ok
            ref[g] = (index, outs, sizes, bounds)
            for k, cpu in enumerate(cpu_ids):
                seg = h.store.get(int(cpu)).segments[g]
                assert seg.components[0].layer_indices == tuple(sel)
                assert seg.compressed_size == sizes[k]
                assert np.float32(seg.actual_error_bound) == np.float32(bounds[k])
                assert torch.equal(seg.payload, outs[k][: sizes[k]].cpu())

        restored = torch.zeros(len(pages), kv[0].numel(), dtype=torch.bfloat16, device="cuda")
        for g in range(2):
            index, outs, sizes, bounds = ref[g]
            assert w.decompress_batch_fixed_bf16_indexed_scatter(
                outs, sizes, list(restored), index, prefix, layers, epl, bounds)
        dst_gpu = np.array([2, 3, 5, 6, 10, 11, 12, 13, 14], dtype=np.int64)   # not sources
        kv[torch.as_tensor(dst_gpu, device="cuda")] = 0
        assert h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids, dst_gpu))
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        for j in range(len(gpu_ids)):
            assert torch.equal(kv[dst_gpu[j]].view(-1).view(torch.int16),
                               restored[j].view(torch.int16))

        slab = h.store.slab(h.store.record(int(cpu_ids[0])).slab).buffer
        dst = [torch.zeros(kv[0].numel(), dtype=torch.bfloat16, device="cuda") for _ in pages]
        t = ko.restore_job(slab, dst, h.engine)
        assert h.engine.lib.ckv_pipe_wait(h.engine.pipe, t) == 0
        for k in range(len(pages)):
            assert torch.equal(dst[k].view(torch.int16), restored[k].view(torch.int16))
    finally:
        h.shutdown()


def _plain_wrapper(cpp, eb):
    cfg = cpp.CompressionConfig(error_bound=eb, use_relative_error=True,
                                processing_dim=cpp.CuszpDim.DIM_1D,
                                encoding_mode=cpp.CuszpMode.MODE_FIXED,
                                data_type=cpp.CuszpType.TYPE_FLOAT)
    return cpp.CuSZpWrapper(cfg, 0)


@pytest.mark.gpu
def test_handlers_store_incompressible_pages_raw():
    """Pages that cuSZp would not shrink below their BF16 size are stored raw
    with bound 0 (vllm_v1_compressed_offload.py:1000-1010) and come back bit
    for bit; the others keep the plain call's bytes."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp as cpp

    shape = (2, 28, 2, 16, 128)
    kv = _kv(16, shape, seed=21).cuda()
    g = torch.Generator().manual_seed(22)
    noisy = [2, 5, 6]
    for b in noisy:   # uniform in [-1, 1]: 15 bits per value at REL 1e-5
        kv[b] = (torch.rand(shape, generator=g) * 2 - 1).to(torch.bfloat16).cuda()
    snapshot = kv.clone()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-5, device_id=0, chunk_pages=4)
    try:
        gpu_ids = np.arange(0, 8, dtype=np.int64)
        cpu_ids = gpu_ids + 500
        h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        w = _plain_wrapper(cpp, 1e-5)
        n = kv[0].numel()
        outs = [torch.empty(w.estimate_compressed_buffer_size(n * 4), dtype=torch.uint8,
                            device="cuda") for _ in gpu_ids]
        ok, sizes, bounds = w.compress_batch_fixed_bf16([kv[i].view(-1) for i in gpu_ids], outs,
                                                        [1e-5] * len(gpu_ids))
        assert ok
        for k, cpu in enumerate(cpu_ids):
            seg = h.store.get(int(cpu)).segments[0]
            if k in noisy:
                assert sizes[k] >= 2 * n
                assert seg.encoding == "raw" and seg.compressed_size == 2 * n
                assert seg.actual_error_bound == 0.0
                assert torch.equal(seg.payload, kv[k].view(-1).view(torch.uint8).cpu())
            else:
                assert seg.encoding == "cuszp" and seg.compressed_size == sizes[k]
                assert torch.equal(seg.payload, outs[k][: sizes[k]].cpu())
        dst = np.arange(8, 16, dtype=np.int64)
        kv[8:16] = 0
        h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids, dst))
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        restored = torch.zeros(len(gpu_ids), n, dtype=torch.bfloat16, device="cuda")
        assert w.decompress_batch_fixed_bf16(outs, sizes, restored, n, bounds)
        torch.cuda.synchronize()
        for k in range(len(gpu_ids)):
            want = snapshot[k].view(-1) if k in noisy else restored[k]
            assert torch.equal(kv[8 + k].view(-1).view(torch.int16), want.view(torch.int16)), k
        # and from the slab bytes alone
        slab = h.store.slab(h.store.record(int(cpu_ids[0])).slab).buffer
        pages = [torch.zeros(n, dtype=torch.bfloat16, device="cuda") for _ in gpu_ids]
        t = ko.restore_job(slab, pages, h.engine)
        assert h.engine.lib.ckv_pipe_wait(h.engine.pipe, t) == 0
        for k in range(len(gpu_ids)):
            assert torch.equal(pages[k].view(torch.int16), kv[8 + k].view(-1).view(torch.int16))
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_pad_small_pages():
    """Pages below 36864 elements are coded zero-padded to 36864, as the
    reference's connector pads them (vllm_v1_compressed_offload.py:904-909):
    the stored bytes equal the plain call on padded pages, the restore its
    first n elements."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp as cpp

    shape = (2, 1, 2, 16, 128)            # one layer's K and V: 8192 elements
    kv = _kv(32, shape, seed=23).cuda()
    n, coded = kv[0].numel(), 36864
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=8)
    try:
        gpu_ids = np.array([1, 3, 5, 7, 9, 11, 13, 15, 17, 19], dtype=np.int64)
        cpu_ids = gpu_ids + 40
        h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        padded = torch.zeros(len(gpu_ids), coded, dtype=torch.bfloat16, device="cuda")
        padded[:, :n] = kv[torch.as_tensor(gpu_ids)].view(len(gpu_ids), -1)
        w = _plain_wrapper(cpp, 1e-4)
        outs = [torch.empty(w.estimate_compressed_buffer_size(coded * 4), dtype=torch.uint8,
                            device="cuda") for _ in gpu_ids]
        ok, sizes, bounds = w.compress_batch_fixed_bf16(list(padded), outs, [1e-4] * len(gpu_ids))
        assert ok
        for k, cpu in enumerate(cpu_ids):
            seg = h.store.get(int(cpu)).segments[0]
            assert seg.encoding == "cuszp" and seg.compressed_numel == coded
            assert seg.compressed_size == sizes[k]
            assert np.float32(seg.actual_error_bound) == np.float32(bounds[k])
            assert torch.equal(seg.payload, outs[k][: sizes[k]].cpu())
        dst = gpu_ids - 1
        kv[torch.as_tensor(dst)] = 0
        h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids, dst))
        h.cpu_to_gpu_handler.wait({2})
        restored = torch.zeros(len(gpu_ids) * coded, dtype=torch.bfloat16, device="cuda")
        assert w.decompress_batch_fixed_bf16(outs, sizes, restored, coded, bounds)
        torch.cuda.synchronize()
        restored = restored.view(len(gpu_ids), coded)[:, :n]
        for k, d in enumerate(dst):
            assert torch.equal(kv[d].view(-1).view(torch.int16), restored[k].view(torch.int16))
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_layer_groups_with_a_raw_segment():
    """A layer segment that does not compress is stored raw; the page's
    other segment keeps the indexed call's bytes; the load restores both."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp as cpp

    shape = (2, 28, 2, 16, 128)
    layers, prefix, epl = 28, 2, 2 * 16 * 128
    low = [0, 1, 2, 5, 19, 20, 21]
    high = [i for i in range(layers) if i not in low]
    kv = _kv(12, shape, seed=24).cuda()
    g = torch.Generator().manual_seed(25)
    # page 1's low-bound layers: uniform noise (incompressible at 1e-5)
    noise = (torch.rand(2, len(low), 2, 16, 128, generator=g) * 2 - 1).to(torch.bfloat16).cuda()
    kv[1][:, low] = noise
    snapshot = kv.clone()
    bounds_of = {i: (1e-5 if i in low else 1e-4) for i in range(layers)}
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=2,
                                              layer_bounds=bounds_of)
    try:
        gpu_ids = np.array([0, 1, 2, 3], dtype=np.int64)
        cpu_ids = gpu_ids + 70
        h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        seg = h.store.get(71).segments[0]
        assert seg.encoding == "raw" and seg.actual_error_bound == 0.0
        assert torch.equal(seg.payload, kv[1][:, low].contiguous().view(-1).view(torch.uint8).cpu())
        assert h.store.get(71).segments[1].encoding == "cuszp"
        assert all(s.encoding == "cuszp" for c in (70, 72, 73) for s in h.store.get(c).segments)

        w = _plain_wrapper(cpp, 1e-4)
        want = torch.zeros(len(gpu_ids), kv[0].numel(), dtype=torch.bfloat16, device="cuda")
        for gi, (eb, sel) in enumerate([(1e-5, low), (1e-4, high)]):
            index = torch.tensor(sel, device="cuda")
            pages = [kv[i].view(-1) for i in gpu_ids]
            outs = [torch.empty(w.estimate_compressed_buffer_size(prefix * len(sel) * epl * 4),
                                dtype=torch.uint8, device="cuda") for _ in pages]
            ok, sizes, bounds = w.compress_batch_fixed_bf16_indexed(
                pages, outs, index, prefix, layers, epl, [eb] * len(pages))
            assert ok
            assert w.decompress_batch_fixed_bf16_indexed_scatter(
                outs, sizes, list(want), index, prefix, layers, epl, bounds)
        torch.cuda.synchronize()
        want[1].view(prefix, layers, epl)[:, low] = snapshot[1].view(prefix, layers, epl)[:, low]
        dst = np.array([8, 9, 10, 11], dtype=np.int64)
        kv[8:12] = 0
        h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids, dst))
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        for k, d in enumerate(dst):
            assert torch.equal(kv[d].view(-1).view(torch.int16), want[k].view(torch.int16)), k
    finally:
        h.shutdown()


@pytest.mark.gpu
@pytest.mark.parametrize("codec", ["int8", "raw"])
def test_handlers_comparison_codecs(codec):
    """The connector's INT8 and raw codecs through the handlers: INT8 pages
    restore to what the reference's torch expression gives on the GPU
    (vllm_v1_compressed_offload.py:711-724, 2090-2116) and carry its scale
    and bound once stored; raw pages restore bit for bit."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    shape = (2, 28, 2, 16, 128)
    kv = _kv(20, shape, seed=31).cuda()
    snapshot = kv.clone()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=4,
                                              codec=codec)
    try:
        gpu_ids = np.arange(0, 10, dtype=np.int64)
        cpu_ids = gpu_ids + 900
        h.gpu_to_cpu_handler.transfer_async(1, (gpu_ids, cpu_ids))
        h.gpu_to_cpu_handler.wait({1})
        assert [r.success for r in h.gpu_to_cpu_handler.get_finished()] == [True]
        x = snapshot[:10].view(10, -1).float()
        if codec == "int8":
            scale = x.abs().amax(dim=1, keepdim=True) / 127.0
            scale = torch.where(scale == 0, torch.ones_like(scale), scale)
            q = torch.clamp(torch.round(x / scale), -127, 127).to(torch.int8)
            want = (q.to(torch.float32) * scale).to(torch.bfloat16)
            for k, cpu in enumerate(cpu_ids):
                seg = h.store.get(int(cpu)).segments[0]
                assert seg.encoding == "int8" and seg.compressed_size == kv[0].numel() + 4
                assert np.float32(seg.quant_scale) == np.float32(scale[k].item())
                assert seg.actual_error_bound == seg.quant_scale / 2.0
                assert torch.equal(seg.payload[:kv[0].numel()].view(torch.int8), q[k].cpu())
        else:
            want = snapshot[:10].view(10, -1)
            for cpu in cpu_ids:
                seg = h.store.get(int(cpu)).segments[0]
                assert seg.encoding == "raw" and seg.compressed_size == 2 * kv[0].numel()
        dst = np.arange(10, 20, dtype=np.int64)
        kv[10:20] = 0
        h.cpu_to_gpu_handler.transfer_async(2, (cpu_ids, dst))
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        assert torch.equal(kv[10:20].view(10, -1).view(torch.int16), want.view(torch.int16))
        slab = h.store.slab(h.store.record(int(cpu_ids[0])).slab).buffer
        pages = [torch.zeros(kv[0].numel(), dtype=torch.bfloat16, device="cuda") for _ in gpu_ids]
        t = ko.restore_job(slab, pages, h.engine)
        assert h.engine.lib.ckv_pipe_wait(h.engine.pipe, t) == 0
        assert torch.equal(torch.stack(pages).view(torch.int16), want.view(torch.int16))
    finally:
        h.shutdown()


@pytest.mark.gpu
def test_handlers_zero_bound_layers_stay_exact():
    """The reference's mixed policy test (tests/test_vllm_v1_compressed_offload.py:654-716):
    layers of bound zero are stored raw and restored exactly, the others within
    their bound; the KV cache is byte storage holding BF16 pages; a page whose
    layers all have bound zero is one raw segment."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    layers, prefix, epl = 24, 2, 2 * 16 * 64
    page_numel = prefix * layers * epl
    backing = torch.randn(3, page_numel, dtype=torch.bfloat16, device="cuda")
    tensor = backing.view(torch.uint8).view(torch.int8).reshape(3, -1)
    expected = backing[0].clone()
    bounds_of = {i: (0.0 if i < 12 else 1e-2) for i in range(layers)}
    h = ko.CompressedCpuGpuOffloadingHandlers(tensor, error_bound=1e-4, device_id=0,
                                              chunk_pages=4, layer_bounds=bounds_of)
    try:
        h.gpu_to_cpu_handler.transfer_async(1, (np.array([0]), np.array([0])))
        h.gpu_to_cpu_handler.wait({1})
        stored = h.gpu_to_cpu_handler.get_finished()[0]
        assert stored.success and stored.transfer_size < page_numel * 2
        segs = h.store.get(0).segments
        assert [s.encoding for s in segs] == ["raw", "cuszp"]
        assert segs[0].components[0].layer_indices == tuple(range(12))
        tensor[1].zero_()
        h.cpu_to_gpu_handler.transfer_async(2, (np.array([0]), np.array([1])))
        h.cpu_to_gpu_handler.wait({2})
        torch.cuda.synchronize()
        got = backing[1].view(prefix, layers, 2, 16, 64)
        want = expected.view(prefix, layers, 2, 16, 64)
        assert torch.equal(got[:, :12], want[:, :12])
        assert torch.isfinite(got[:, 12:]).all()
        assert torch.allclose(got[:, 12:].float(), want[:, 12:].float(), atol=0.12, rtol=0.12)
    finally:
        h.shutdown()
    green = ko.CompressedCpuGpuOffloadingHandlers(tensor, error_bound=1e-4, device_id=0,
                                                  layer_bounds={i: 0.0 for i in range(layers)})
    try:
        green.gpu_to_cpu_handler.transfer_async(1, (np.array([2]), np.array([5])))
        green.gpu_to_cpu_handler.wait({1})
        segs = green.store.get(5).segments
        assert len(segs) == 1 and segs[0].encoding == "raw"
        assert segs[0].components[0].layer_axis is None
        assert torch.equal(segs[0].payload, tensor[2].view(torch.uint8).cpu())
    finally:
        green.shutdown()


@pytest.mark.gpu
def test_handlers_many_jobs_polled_from_another_thread():
    """More jobs than the pipeline's 64 ticket events, with finished jobs
    polled from a second thread while the first submits them (the reference
    runs its stores on a worker thread, vllm_v1_compressed_offload.py:2365-2385):
    every job reports success once, and the pages stored first -- whose store
    tickets have retired before their loads are issued -- restore bit for bit
    as the plain calls restore them."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import threading
    import time

    import cuszp_wrapper_cpp as cpp

    jobs, shape = 70, (2, 8, 2, 16, 128)
    kv = _kv(2 * jobs, shape, seed=14).cuda()
    kv[jobs:].zero_()   # rate-0 blocks are not written on restore
    n = kv[0].numel()
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=1e-4, device_id=0, chunk_pages=4)
    results: dict[int, list[bool]] = {}
    submitted = threading.Event()

    def poll():
        deadline = time.monotonic() + 120
        while time.monotonic() < deadline:
            for handler in (h.gpu_to_cpu_handler, h.cpu_to_gpu_handler):
                for r in handler.get_finished():
                    results.setdefault(r.job_id, []).append(r.success)
            if submitted.is_set() and len(results) == 2 * jobs:
                return
            time.sleep(1e-4)

    poller = threading.Thread(target=poll)
    poller.start()
    try:
        for i in range(jobs):
            assert h.gpu_to_cpu_handler.transfer_async(i, (np.array([i]), np.array([1000 + i])))
        for i in range(jobs):
            assert h.cpu_to_gpu_handler.transfer_async(
                jobs + i, (np.array([1000 + i]), np.array([jobs + i])))
    finally:
        submitted.set()
        poller.join(timeout=150)
    try:
        assert not poller.is_alive()
        assert results == {j: [True] for j in range(2 * jobs)}
        torch.cuda.synchronize()
        cfg = cpp.CompressionConfig(error_bound=1e-4, use_relative_error=True,
                                    processing_dim=cpp.CuszpDim.DIM_1D,
                                    encoding_mode=cpp.CuszpMode.MODE_FIXED,
                                    data_type=cpp.CuszpType.TYPE_FLOAT)
        w = cpp.CuSZpWrapper(cfg, 0)
        pages = [kv[i].view(-1) for i in range(jobs)]
        outs = [torch.empty(w.estimate_compressed_buffer_size(n * 4), dtype=torch.uint8,
                            device="cuda") for _ in pages]
        ok, sizes, bounds = w.compress_batch_fixed_bf16(pages, outs, [1e-4] * jobs)
        assert ok
        ref = torch.zeros(jobs * n, dtype=torch.bfloat16, device="cuda")
        assert w.decompress_batch_fixed_bf16(outs, sizes, ref, n, bounds)
        torch.cuda.synchronize()
        assert torch.equal(kv[jobs:].reshape(-1).view(torch.int16), ref.view(torch.int16))
    finally:
        h.shutdown()


def test_job_header_round_trips_any_layout():
    """Write / read of the job format over random layouts: page counts, layer
    groups (including raw zero-bound ones), raw entries and codecs."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=60, deadline=None)
    @given(st.integers(1, 9), st.integers(1, 4), st.integers(2, 30), st.integers(0, 2**31),
           st.sampled_from(["cuszp", "int8", "raw"]))
    def check(count, segs, layers, seed, codec):
        rng = np.random.default_rng(seed)
        if codec != "cuszp":
            segs = 1
        segs = min(segs, layers)
        prefix, epl = 2, 64
        n = prefix * layers * epl
        groups = None
        if segs > 1:
            owner = rng.permutation(np.arange(layers) % segs)
            groups = [(float(g) * 1e-4, tuple(int(x) for x in np.flatnonzero(owner == g)))
                      for g in range(segs)]
        seg_elems = [n] if groups is None else [prefix * len(sel) * epl for _b, sel in groups]
        entries = count * segs
        raw = (rng.random(entries) < 0.3) if codec == "cuszp" else np.full(entries, codec == "raw")
        sizes, offsets, pos = [], [], 0
        for j in range(entries):
            full = 2 * seg_elems[j % segs]
            if codec == "int8":
                size = (n + 3) // 4 * 4 + 4
            elif raw[j]:
                size = full
            else:
                size = int(rng.integers(1, full))
            offsets.append(pos)
            sizes.append(size)
            pos += (size + 15) // 16 * 16
        bounds = rng.random(entries).astype(np.float32)
        hdr = ko.JobHeader.bytes_for(count, segs, layers if segs > 1 else 0)
        slab = torch.zeros(hdr + pos, dtype=torch.uint8)
        ko.JobHeader.write(slab, n, 1e-4, True, (C.c_size_t * entries)(*offsets),
                           (C.c_size_t * entries)(*sizes), (C.c_float * entries)(*bounds.tolist()),
                           pos, groups, prefix, layers if segs > 1 else 0, raw=raw.tolist(),
                           codec=codec)
        job = ko.JobHeader.read(slab)
        assert job["count"] == count and job["segments"] == segs and job["codec"] == codec
        assert job["sizes"].tolist() == sizes and job["offsets"].tolist() == offsets
        assert job["bounds"].tolist() == bounds.tolist()
        assert job["raw"].tolist() == raw.tolist()
        if groups is not None:
            assert [sel for _b, sel in job["groups"]] == [sel for _b, sel in groups]

    check()
