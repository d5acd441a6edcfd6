"""The reference's comparison codecs (INT8, vllm_v1_compressed_offload.py:711-724
and :2090-2116; raw, :1578-1615) through the store / restore pipeline, on the
GPU: stored bytes against the numpy oracle and the reference's torch
expression on the same device, restores bit for bit, overlapped jobs."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import int8_codec as oc

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
    cfg = _ckv.Config(1e-4, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
    assert lib.ckv_create(cfg, 0, C.byref(ctx)) == 0
    yield _ckv, lib, ctx
    lib.ckv_destroy(ctx)


def _torch_reference(page):
    x = page.to(torch.float32)
    scale_t = x.abs().max() / 127.0
    if float(scale_t.item()) == 0.0:
        scale_t = torch.ones_like(scale_t)
    q = torch.clamp(torch.round(x / scale_t), -127, 127).to(torch.int8)
    out = (q.to(torch.float32) * float(scale_t.item())).to(torch.bfloat16)
    return q, float(scale_t.item()), out


@pytest.mark.parametrize("count,n,chunk", [(37, 229376, 8), (5, 40001, 2), (64, 8192, 64),
                                           (3, 1000, 7)])
def test_int8_pipe_matches_oracle_and_torch(env, count, n, chunk):
    _ckv, lib, ctx = env
    pages = _pages(count, n, seed=count + n)
    pages[1 % count].zero_()                      # an all-zero page: scale 1
    dev = pages.cuda()
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, chunk, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity_int8(count, n))
        host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        sizes = (C.c_size_t * count)()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        s = torch.cuda.current_stream().cuda_stream
        ptrs = _ckv.ptr_array([dev[i].data_ptr() for i in range(count)])
        assert lib.ckv_pipe_store_int8(pipe, ptrs, count, n, host.data_ptr(), cap, offsets, sizes,
                                       C.byref(total), 0, C.byref(ticket), s) == 0
        assert lib.ckv_pipe_wait(pipe, ticket.value) == 0
        assert total.value <= cap
        bits = pages.view(torch.int16).numpy().view(np.uint16)
        for i in range(count):
            q, scale = oc.encode(bits[i])
            assert offsets[i] % 16 == 0 and sizes[i] == oc.align4(n) + 4
            got = bytes(host[offsets[i]:offsets[i] + sizes[i]].numpy())
            assert got == oc.stored_page(q, scale), f"page {i}"
            tq, tscale, _ = _torch_reference(dev[i])
            assert np.float32(tscale) == scale
            assert torch.equal(tq.cpu(), torch.from_numpy(q))
        restored = torch.full_like(dev, 3.0)
        t2 = C.c_uint64(0)
        assert lib.ckv_pipe_restore_int8(
            pipe, host.data_ptr(), offsets, count, n,
            _ckv.ptr_array([restored[i].data_ptr() for i in range(count)]), ticket.value,
            C.byref(t2), s) == 0
        torch.cuda.synchronize()
        for i in range(count):
            q, scale = oc.encode(bits[i])
            want = oc.decode(q, scale)
            assert np.array_equal(restored[i].view(torch.int16).cpu().numpy().view(np.uint16), want)
            assert torch.equal(restored[i].view(torch.int16), _torch_reference(dev[i])[2].view(torch.int16))
    finally:
        lib.ckv_pipe_destroy(pipe)


@pytest.mark.parametrize("count,page_bytes,chunk", [(33, 458752, 8), (4, 1002, 3)])
def test_raw_pipe_round_trip(env, count, page_bytes, chunk):
    _ckv, lib, ctx = env
    g = torch.Generator().manual_seed(page_bytes)
    src = torch.randint(0, 256, (count, page_bytes), generator=g, dtype=torch.uint8).cuda()
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, chunk, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity_raw(count, page_bytes))
        host = torch.zeros(cap, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ckv_pipe_store_raw(pipe, _ckv.ptr_array([src[i].data_ptr() for i in range(count)]),
                                      count, page_bytes, host.data_ptr(), cap, offsets,
                                      C.byref(total), 0, C.byref(ticket), s) == 0
        dst = torch.zeros_like(src)
        t2 = C.c_uint64(0)
        assert lib.ckv_pipe_restore_raw(pipe, host.data_ptr(), offsets, count, page_bytes,
                                        _ckv.ptr_array([dst[i].data_ptr() for i in range(count)]),
                                        ticket.value, C.byref(t2), s) == 0
        torch.cuda.synchronize()
        cpu = src.cpu()
        for i in range(count):
            assert torch.equal(host[offsets[i]:offsets[i] + page_bytes], cpu[i])
        assert torch.equal(dst, src)
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_int8_pipe_special_values(env):
    """Pages with NaN, with Inf, and with subnormal-scale values: stored bytes
    and restores equal the reference's expression on CUDA tensors."""
    _ckv, lib, ctx = env
    count, n = 4, 4096
    pages = _pages(count, n, seed=77)
    pages[0, 17] = float("nan")
    pages[1, 5] = float("inf")
    pages[1, 9] = float("-inf")
    pages[2] = pages[2] * 1e-38
    dev = pages.cuda()
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 2, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity_int8(count, n))
        host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        sizes = (C.c_size_t * count)()
        total = C.c_size_t(0)
        t1, t2 = C.c_uint64(0), C.c_uint64(0)
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ckv_pipe_store_int8(pipe, _ckv.ptr_array([dev[i].data_ptr() for i in range(count)]),
                                       count, n, host.data_ptr(), cap, offsets, sizes,
                                       C.byref(total), 0, C.byref(t1), s) == 0
        restored = torch.zeros_like(dev)
        assert lib.ckv_pipe_restore_int8(pipe, host.data_ptr(), offsets, count, n,
                                         _ckv.ptr_array([restored[i].data_ptr() for i in range(count)]),
                                         t1.value, C.byref(t2), s) == 0
        torch.cuda.synchronize()
        for i in range(count):
            tq, tscale, tout = _torch_reference(dev[i])
            q = torch.frombuffer(bytearray(bytes(host[offsets[i]:offsets[i] + n].numpy())),
                                 dtype=torch.int8)
            assert torch.equal(q, tq.cpu()), f"page {i}"
            assert torch.equal(restored[i].view(torch.int16), tout.view(torch.int16)), f"page {i}"
            oq, oscale = oc.encode(pages[i].view(torch.int16).numpy().view(np.uint16))
            assert np.array_equal(oq, q.numpy())
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_int8_pipe_overlapped_jobs(env):
    """Step k stores into slab k % 2 while step k-1's slab is restored."""
    _ckv, lib, ctx = env
    count, n = 40, 65536
    batches = [_pages(count, n, seed=300 + k).cuda() for k in range(4)]
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 16, C.byref(pipe)) == 0
    try:
        cap = int(lib.ckv_pipe_host_capacity_int8(count, n))
        slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * count)(), "s": (C.c_size_t * count)(), "t": C.c_size_t(0)}
                for _ in range(2)]
        s = torch.cuda.current_stream().cuda_stream
        t_store = t_rest = 0
        outs = []
        for k in range(len(batches) + 1):
            ts = C.c_uint64(0)
            if k < len(batches):
                a = meta[k % 2]
                ptrs = _ckv.ptr_array([batches[k][i].data_ptr() for i in range(count)])
                assert lib.ckv_pipe_store_int8(pipe, ptrs, count, n, slabs[k % 2].data_ptr(), cap,
                                               a["o"], a["s"], C.byref(a["t"]), t_rest,
                                               C.byref(ts), s) == 0
            if k > 0:
                b = meta[(k + 1) % 2]
                out = torch.empty(count, n, dtype=torch.bfloat16, device="cuda")
                tr = C.c_uint64(0)
                assert lib.ckv_pipe_restore_int8(
                    pipe, slabs[(k + 1) % 2].data_ptr(), b["o"], count, n,
                    _ckv.ptr_array([out[i].data_ptr() for i in range(count)]), t_store,
                    C.byref(tr), s) == 0
                t_rest = tr.value
                outs.append(out)
            t_store = ts.value
        torch.cuda.synchronize()
        for k, out in enumerate(outs):
            for i in range(count):
                assert torch.equal(out[i].view(torch.int16),
                                   _torch_reference(batches[k][i])[2].view(torch.int16)), (k, i)
    finally:
        lib.ckv_pipe_destroy(pipe)


def test_int8_pipe_rejects_small_host_buffer(env):
    _ckv, lib, ctx = env
    count, n = 4, 32768
    dev = _pages(count, n, seed=9).cuda()
    pipe = C.c_void_p()
    assert lib.ckv_pipe_create(ctx, 2, C.byref(pipe)) == 0
    try:
        host = torch.empty(1024, dtype=torch.uint8, pin_memory=True)
        offsets = (C.c_size_t * count)()
        sizes = (C.c_size_t * count)()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        st = lib.ckv_pipe_store_int8(pipe, _ckv.ptr_array([dev[i].data_ptr() for i in range(count)]),
                                     count, n, host.data_ptr(), host.numel(), offsets, sizes,
                                     C.byref(total), 0, C.byref(ticket),
                                     torch.cuda.current_stream().cuda_stream)
        assert st == 4  # CKV_ERR_CAPACITY
        torch.cuda.synchronize()
    finally:
        lib.ckv_pipe_destroy(pipe)
