"""The two BF16 encoders against each other (GPU).

libckv has a clustered encoder (a unit spread over a thread-block cluster,
read once) and a streaming one (one unit per CTA, read twice); the automatic
choice takes the streaming encoder for whole pages of at most 16384
elements.  Forced through ckv_set_encoder on the same pages, both must give
identical sizes, bounds and compressed bytes -- which the golden and oracle
parity tests then pin to the reference for either choice -- for every unit
size around the chunk (8192 elements) and block (32) boundaries, relative
and absolute bounds, specials (NaN, infinities, subnormals, constant and
zero pages) and blocks whose |q| reaches 2^15 (the exact quantiser's path).
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CLUSTER, STREAM = 1, 2


def _pages(count, n, seed, kind):
    g = torch.Generator().manual_seed(seed)
    if kind == "kv":
        scale = torch.empty(128).log_normal_(0.0, 0.5, generator=g)
        x = torch.randn(count, n, generator=g) * scale.repeat(n // 128 + 1)[:n]
    elif kind == "one_sided":   # |q| up to 2^16 at REL 1e-5: wide blocks
        x = torch.rand(count, n, generator=g) * 10.0 + 5.0
    elif kind == "specials":
        x = torch.randn(count, n, generator=g)
        vals = torch.tensor([float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1e-40,
                             -1e-40, 3e38, -3e38])
        idx = torch.randint(0, n, (count, max(1, n // 97)), generator=g)
        x.scatter_(1, idx, vals[torch.randint(0, len(vals), idx.shape, generator=g)])
    elif kind == "const":
        x = torch.full((count, n), 1.5)
    elif kind == "zero":
        x = torch.zeros(count, n)
    else:
        raise ValueError(kind)
    return x.to(torch.bfloat16)


def _compress(lib, _ckv, pages, eb, relative, choice, cap, fill=0xA5):
    count, n = pages.shape
    dev = pages.device
    out = torch.full((count, cap + 64), fill, dtype=torch.uint8, device=dev)
    ctx = C.c_void_p()
    cfg = _ckv.Config(eb, 1 if relative else 0, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
    assert lib.ckv_create(cfg, 0, C.byref(ctx)) == 0
    try:
        assert lib.ckv_set_encoder(ctx, choice) == 0
        sizes = (C.c_size_t * count)()
        bounds = (C.c_float * count)()
        status = lib.ckv_compress_batch_fixed_bf16(
            ctx, _ckv.ptr_array([pages[i].data_ptr() for i in range(count)]),
            _ckv.ptr_array([out[i].data_ptr() for i in range(count)]), None, count, n, cap,
            sizes, bounds, torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize(dev)
    finally:
        lib.ckv_destroy(ctx)
    return status, list(sizes), [C.c_float(b).value for b in bounds], out


def _capacity(lib, n):
    """The reference's buffer estimate, or the worst case where a tiny unit's
    1024-byte header alone exceeds it."""
    from oracle.oracle import capacity_for

    return max(int(lib.ckv_estimate_compressed_buffer_size(n * 4)), capacity_for(n))


@pytest.fixture(scope="module")
def lib_ckv():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import _ckv

    torch.cuda.set_device(0)
    return _ckv.load(), _ckv


CASES = [(n, kind, eb, rel) for n in (1, 31, 32, 33, 1000, 8191, 8192, 8193, 16384, 16385, 24576,
                                      40001, 229376)
         for kind, eb, rel in (("kv", 1e-4, True), ("kv", 1e-5, True), ("kv", 2e-3, False))]
CASES += [(n, kind, 1e-5, True) for n in (4096, 16384, 40001)
          for kind in ("one_sided", "specials", "const", "zero")]
CASES += [(8192, "specials", 1e-3, False), (16384, "one_sided", 1e-4, False)]
# C5 and C4 page sizes (the clustered encoder's 100 KB slice geometry)
CASES += [(327680, "kv", 1e-4, True), (458752, "kv", 1e-5, True)]


@pytest.mark.parametrize("n,kind,eb,relative", CASES)
def test_streaming_and_clustered_encoders_write_the_same_bytes(lib_ckv, n, kind, eb, relative):
    lib, _ckv = lib_ckv
    pages = _pages(6, n, seed=n * 7 + len(kind), kind=kind).cuda()
    cap = _capacity(lib, n)
    s1, sizes1, bounds1, out1 = _compress(lib, _ckv, pages, eb, relative, CLUSTER, cap)
    s2, sizes2, bounds2, out2 = _compress(lib, _ckv, pages, eb, relative, STREAM, cap)
    assert s1 == 0 and s2 == 0
    assert sizes1 == sizes2
    assert np.array_equal(np.array(bounds1, np.float32).view(np.uint32),
                          np.array(bounds2, np.float32).view(np.uint32))
    for i, s in enumerate(sizes1):
        assert torch.equal(out1[i, :s], out2[i, :s]), f"unit {i}"
        # nothing written past the reported size
        assert bool((out2[i, s:] == 0xA5).all()), f"unit {i}"


def test_automatic_choice_matches_both(lib_ckv):
    """AUTO on small whole pages (streaming) and on large ones (clustered)."""
    lib, _ckv = lib_ckv
    for n in (8192, 229376):
        pages = _pages(8, n, seed=3, kind="kv").cuda()
        cap = _capacity(lib, n)
        ref = _compress(lib, _ckv, pages, 1e-4, True, CLUSTER, cap)
        auto = _compress(lib, _ckv, pages, 1e-4, True, 0, cap)
        assert auto[0] == 0 and auto[1] == ref[1] and auto[2] == ref[2]
        for i, s in enumerate(ref[1]):
            assert torch.equal(ref[3][i, :s], auto[3][i, :s])


@pytest.mark.parametrize("count,n", [(256, 229376), (271, 229376), (256, 327680), (512, 327680)])
def test_remainder_units_on_the_streaming_kernel(lib_ckv, count, n):
    """Large batches whose last clustered round would hold a few units alone
    hand those units to the streaming encoder, launched beside the clustered
    one: the automatic choice writes the bytes of the clustered encoder."""
    lib, _ckv = lib_ckv
    pages = _pages(count, n, seed=count, kind="kv").cuda()
    cap = _capacity(lib, n)
    ref = _compress(lib, _ckv, pages, 1e-5, True, CLUSTER, cap)
    auto = _compress(lib, _ckv, pages, 1e-5, True, 0, cap)
    assert ref[0] == 0 and auto[0] == 0
    assert auto[1] == ref[1] and auto[2] == ref[2]
    for i, s in enumerate(ref[1]):
        assert torch.equal(ref[3][i, :s], auto[3][i, :s]), f"unit {i}"


def test_unaligned_pages_take_the_clustered_encoder(lib_ckv):
    """Pages that do not start on 16 bytes are not whole pages: forcing the
    streaming encoder falls back to the clustered one, same bytes."""
    lib, _ckv = lib_ckv
    n = 8192
    base = _pages(4, n + 8, seed=11, kind="kv").cuda()
    pages = base[:, 1:n + 1]                  # 2-byte offset, rows still strided
    cap = _capacity(lib, n)
    contiguous = pages.contiguous()
    ref = _compress(lib, _ckv, contiguous, 1e-4, True, CLUSTER, cap)
    forced = _compress(lib, _ckv, pages, 1e-4, True, STREAM, cap)
    assert forced[0] == 0 and forced[1] == ref[1] and forced[2] == ref[2]
    for i, s in enumerate(ref[1]):
        assert torch.equal(ref[3][i, :s], forced[3][i, :s])


def test_capacity_overflow_on_both_encoders(lib_ckv):
    """Units whose 1024-byte header alone exceeds the smallest buffer the
    batch entry point accepts (8 bytes an element): CKV_ERR_CAPACITY from
    both encoders, the needed size reported, nothing written past the
    buffer."""
    lib, _ckv = lib_ckv
    for n in (16, 100):
        pages = _pages(3, n, seed=5, kind="kv").cuda()
        full = _compress(lib, _ckv, pages, 1e-5, True, CLUSTER, _capacity(lib, n))
        assert full[0] == 0
        cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
        assert cap < min(full[1])
        for choice in (CLUSTER, STREAM):
            status, sizes, _bounds, out = _compress(lib, _ckv, pages, 1e-5, True, choice, cap)
            assert status == 4                   # CKV_ERR_CAPACITY
            assert sizes == full[1]
            assert bool((out[:, cap:] == 0xA5).all())


def test_set_encoder_rejects_unknown_choices(lib_ckv):
    lib, _ckv = lib_ckv
    ctx = C.c_void_p()
    cfg = _ckv.Config(1e-4, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
    assert lib.ckv_create(cfg, 0, C.byref(ctx)) == 0
    try:
        assert lib.ckv_set_encoder(ctx, 3) == 1
        assert lib.ckv_set_encoder(ctx, -1) == 1
        assert lib.ckv_set_encoder(ctx, 2) == 0
    finally:
        lib.ckv_destroy(ctx)
