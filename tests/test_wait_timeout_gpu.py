"""A bounded wait in the encoder runs out, on the GPU, without a fault.

The reference's kernels wait for each other without a limit (their
decoupled look-back spins, cuszp_batched_fixed.cu:241-297).  Every wait in
libckv's encoder is bounded.  Here one cluster of an encode launch is made
to wait for a bound exchange that never comes (ckv_test_withhold_exchange:
the cluster's first CTA sends nothing for one unit, and that cluster's waits
give up after a few thousand polls).  The launch must then

* fail with CKV_ERR_CUDA and the timeout message, quickly;
* mark CKV_DEV_TIMEOUT on exactly the units of that cluster (an arithmetic
  progression through the withheld unit: a cluster walks units first,
  first + clusters, ...) and leave every other unit's bytes, size and bound
  identical to a normal launch;
* leave the context usable: the next normal call gives the same bytes as
  before, which match the C oracle.

No kernel faults, traps or spins without a limit: a wait that runs out sets
a status bit and returns.
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CKV_ERR_CUDA = 3
CKV_DEV_TIMEOUT = 8


def _pages(count, n, seed):
    g = torch.Generator().manual_seed(seed)
    scale = torch.empty(128).log_normal_(0.0, 0.5, generator=g)
    x = torch.randn(count, n, generator=g) * scale.repeat(n // 128 + 1)[:n]
    return x.to(torch.bfloat16)


def _compress(lib, ctx, inputs, outputs, count, n, cap, stream):
    sizes = (C.c_size_t * count)()
    bounds = (C.c_float * count)()
    st = lib.ckv_compress_batch_fixed_bf16(ctx, inputs, outputs, None, count, n, cap, sizes,
                                           bounds, stream)
    return st, list(sizes), [C.c_float(b).value for b in bounds]


def test_withheld_exchange_times_out_and_context_recovers():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv
    from oracle.oracle import COracle

    lib = _ckv.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    count, n, eb, withheld = 64, 229376, 1e-5, 20
    host = _pages(count, n, seed=31)
    pages = host.to(dev)
    cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
    stream = torch.cuda.current_stream(dev).cuda_stream
    inputs = _ckv.ptr_array([pages[i].data_ptr() for i in range(count)])
    ctx = C.c_void_p()
    assert lib.ckv_create(_ckv.Config(eb, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT), 0,
                          C.byref(ctx)) == 0
    try:
        outs = [torch.full((count, cap), 0xAB, dtype=torch.uint8, device=dev) for _ in range(3)]
        ptrs = [_ckv.ptr_array([o[i].data_ptr() for i in range(count)]) for o in outs]

        st, sizes0, bounds0 = _compress(lib, ctx, inputs, ptrs[0], count, n, cap, stream)
        assert st == 0

        assert lib.ckv_test_withhold_exchange(ctx, withheld, 4096) == 0
        t0 = time.monotonic()
        st, sizes1, bounds1 = _compress(lib, ctx, inputs, ptrs[1], count, n, cap, stream)
        elapsed = time.monotonic() - t0
        assert st == CKV_ERR_CUDA
        assert b"bounded wait" in lib.ckv_last_error(ctx)
        assert elapsed < 10.0, f"the failed launch took {elapsed:.1f} s"
        status = (C.c_uint32 * count)()
        assert lib.ckv_unit_status(ctx, count, status) == 0
        timed_out = [u for u in range(count) if status[u] & CKV_DEV_TIMEOUT]
        assert withheld in timed_out
        assert all(status[u] == 0 for u in range(count) if u not in timed_out)
        # the units of one cluster: first, first + clusters, ... through the withheld unit
        step = timed_out[1] - timed_out[0] if len(timed_out) > 1 else count
        assert timed_out == list(range(withheld % step, count, step)), timed_out
        assert len(timed_out) < count
        for u in range(count):
            if u in timed_out:
                continue
            assert sizes1[u] == sizes0[u] and bounds1[u] == bounds0[u], u
            assert torch.equal(outs[1][u, : sizes0[u]], outs[0][u, : sizes0[u]]), u

        # the context still works: a normal call gives the same bytes again
        st, sizes2, bounds2 = _compress(lib, ctx, inputs, ptrs[2], count, n, cap, stream)
        assert st == 0 and sizes2 == sizes0 and bounds2 == bounds0
        assert torch.equal(outs[2], outs[0])
        assert lib.ckv_unit_status(ctx, count, status) == 0
        assert not any(status[u] for u in range(count))
        co = COracle()
        bits = host.view(torch.int16).numpy().view(np.uint16)
        for u in (withheld, (withheld + 1) % count):
            ref, ref_eb = co.encode(bits[u], eb, relative=True)
            assert sizes2[u] == ref.size
            assert np.float32(ref_eb).tobytes() == np.float32(bounds2[u]).tobytes()
            assert np.array_equal(outs[2][u, : sizes2[u]].cpu().numpy(), ref), u
    finally:
        lib.ckv_destroy(ctx)
