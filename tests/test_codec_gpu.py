"""Parity of the sm_100a codec (libckv through cuszp_wrapper_cpp) on a GPU.

* against the golden vectors of the reference's own kernels
  (tests/golden/fixtures): compressed bytes, sizes and resolved bounds
  byte-identical; decoded BF16 bit-identical, including the blocks the
  reference decoder leaves untouched (destinations prefilled with a
  sentinel), for the per-page scatter, multi-destination scatter,
  contiguous and layer-indexed modes;
* against the C oracle at larger and random sizes (bit-exact);
* size-independent properties at the benchmark's full size (round trip
  within eb*1.01 + 1e-7 plus one BF16 ulp, re-encode idempotence);
* the API's error behaviour (False, never an exception).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "fixtures"


@pytest.fixture(scope="module")
def cpp():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import cuszp_wrapper_cpp
    return cuszp_wrapper_cpp


@pytest.fixture(scope="module")
def co():
    from oracle.oracle import COracle
    return COracle()


def make_wrapper(cpp, eb=1e-4, relative=True):
    cfg = cpp.CompressionConfig(
        error_bound=eb, use_relative_error=relative,
        processing_dim=cpp.CuszpDim.DIM_1D, encoding_mode=cpp.CuszpMode.MODE_FIXED,
        data_type=cpp.CuszpType.TYPE_FLOAT)
    return cpp.CuSZpWrapper(cfg, 0)


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).cuda().view(torch.bfloat16)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def bf16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    na = (a & 0x7FFF) > 0x7F80
    nb = (b & 0x7FFF) > 0x7F80
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na], b[~nb]))


def golden(name):
    from cases import CASE_BY_NAME
    manifest = json.loads((FIX / "manifest.json").read_text())
    return CASE_BY_NAME[name], np.load(FIX / f"{name}.npz"), manifest["sentinel"]


def encode_case(cpp, case):
    from cases import unit_bits
    w = make_wrapper(cpp, relative=case.relative)
    pages = [bf16_from_bits(unit_bits(case, u)) for u in range(case.batch)]
    # 8 * n bytes (the reference's precondition) is below the 1024-byte header
    # for tiny units; give every unit its worst-case size as well.
    from oracle.oracle import capacity_for
    cap = max(int(w.estimate_compressed_buffer_size(case.n * 4)), capacity_for(case.n))
    outs = [torch.full((cap,), 0xAB, dtype=torch.uint8, device="cuda") for _ in pages]
    eps = [case.eps_of(u) for u in range(case.batch)]
    if case.layer_indices is None:
        ok, sizes, bounds = w.compress_batch_fixed_bf16(pages, outs, eps)
    else:
        idx = torch.tensor(case.layer_indices, dtype=torch.int64, device="cuda")
        ok, sizes, bounds = w.compress_batch_fixed_bf16_indexed(
            pages, outs, idx, case.prefix_count, case.source_layers,
            case.elements_per_layer, eps)
    return w, ok, sizes, bounds, outs


ALL_CASES = [p.stem for p in sorted(FIX.glob("*.npz"))]


@pytest.mark.parametrize("name", ALL_CASES)
def test_encode_matches_reference_goldens(cpp, name):
    case, z, _ = golden(name)
    w, ok, sizes, bounds, outs = encode_case(cpp, case)
    assert ok
    assert [int(s) for s in sizes] == [int(s) for s in z["sizes"]]
    assert np.array_equal(np.array(bounds, dtype=np.float32).view(np.uint32),
                          z["bounds"].astype(np.float32).view(np.uint32))
    off = 0
    for u in range(case.batch):
        s = int(z["sizes"][u])
        got = outs[u][:s].cpu().numpy()
        assert np.array_equal(got, z["compressed"][off:off + s]), f"unit {u}"
        off += s
    # nothing written past the reported size
    for u in range(case.batch):
        tail = outs[u][int(sizes[u]):int(sizes[u]) + 64].cpu().numpy()
        assert np.all(tail == 0xAB)


def _golden_streams(case, z):
    streams = []
    off = 0
    for u in range(case.batch):
        s = int(z["sizes"][u])
        streams.append(torch.from_numpy(z["compressed"][off:off + s].copy()).cuda())
        off += s
    return streams


@pytest.mark.parametrize("name", ALL_CASES)
def test_decode_matches_reference_goldens(cpp, name):
    case, z, sentinel = golden(name)
    w = make_wrapper(cpp)
    streams = _golden_streams(case, z)
    sizes = [int(s) for s in z["sizes"]]
    bounds = [float(b) for b in z["bounds"]]
    if case.layer_indices is not None:
        idx = torch.tensor(case.layer_indices, dtype=torch.int64, device="cuda")
        dests = [torch.full((case.source_numel,), sentinel, dtype=torch.int16,
                            device="cuda").view(torch.bfloat16) for _ in streams]
        assert w.decompress_batch_fixed_bf16_indexed_scatter(
            streams, sizes, dests, idx, case.prefix_count, case.source_layers,
            case.elements_per_layer, bounds)
        torch.cuda.synchronize()
        for u in range(case.batch):
            assert bf16_equal(bits_of(dests[u]), z["decoded"][u])
        return
    per = case.destinations_per_page
    epd = case.n // per
    dests = [torch.full((epd,), sentinel, dtype=torch.int16, device="cuda")
             .view(torch.bfloat16) for _ in range(case.batch * per)]
    assert w.decompress_batch_fixed_bf16_scatter(streams, sizes, dests, case.n, per, epd,
                                                 bounds)
    torch.cuda.synchronize()
    got = np.concatenate([bits_of(d) for d in dests]).reshape(case.batch, case.n)
    for u in range(case.batch):
        assert bf16_equal(got[u], z["decoded"][u])
    # contiguous [batch][n] mode, any n (the reference's pair stores need even n)
    out = torch.full((case.batch * case.n,), sentinel, dtype=torch.int16,
                     device="cuda").view(torch.bfloat16)
    assert w.decompress_batch_fixed_bf16(streams, sizes, out, case.n, bounds)
    torch.cuda.synchronize()
    cont = bits_of(out).reshape(case.batch, case.n)
    for u in range(case.batch):
        assert bf16_equal(cont[u], z["decoded"][u])


def test_non_default_stream(cpp):
    """Same bytes on a side stream (the reference's connector avoids
    non-default streams, vllm_v1_compressed_offload.py:2369-2371)."""
    case, z, _ = golden("min_cuszp")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        w, ok, sizes, bounds, outs = encode_case(cpp, case)
    s.synchronize()
    assert ok and [int(x) for x in sizes] == [int(x) for x in z["sizes"]]
    assert np.array_equal(outs[0][: sizes[0]].cpu().numpy(), z["compressed"][: sizes[0]])


def _kv_pages(n, count, seed):
    g = torch.Generator().manual_seed(seed)
    scale = torch.empty(128).log_normal_(0.0, 0.5, generator=g)
    scale[torch.randperm(128, generator=g)[:4]] *= 8.0
    x = torch.randn(count, n, generator=g) * scale.repeat(n // 128 + 1)[:n]
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("n,count,eb", [
    (229376, 6, 1e-5),     # Qwen2.5-1.5B page (7 groups, cluster of 7)
    (458752, 2, 1e-5),     # Qwen2.5-7B page (14 groups, non-portable cluster)
    (327680, 2, 1e-4),     # Llama-3-70B TP8 page (10 groups)
    (172032, 3, 1e-4),     # 21-layer group of the mixed profile
    (57344, 5, 1e-5),      # 7-layer group
    (8192, 33, 1e-4),      # one layer's K+V
    (524288, 1, 1e-3),     # largest unit of three 64 KB slices per CTA
    (600001, 2, 1e-4),     # two 100 KB slices per CTA, ragged last block
    (819200, 1, 1e-3),     # largest unit of the single-pass encoder
])
def test_encode_decode_match_oracle(cpp, co, n, count, eb):
    host = _kv_pages(n, count, seed=n + count)
    bits = host.view(torch.int16).numpy().view(np.uint16)
    pages = [host[i].cuda() for i in range(count)]
    w = make_wrapper(cpp, eb)
    cap = int(w.estimate_compressed_buffer_size(n * 4))
    outs = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in pages]
    ok, sizes, bounds = w.compress_batch_fixed_bf16(pages, outs, [eb] * count)
    assert ok
    for i in range(count):
        ref, ref_eb = co.encode(bits[i], eb, relative=True)
        assert np.float32(bounds[i]).tobytes() == np.float32(ref_eb).tobytes()
        assert sizes[i] == ref.size
        assert np.array_equal(outs[i][: sizes[i]].cpu().numpy(), ref)
    dest = torch.zeros(count * n, dtype=torch.bfloat16, device="cuda")
    assert w.decompress_batch_fixed_bf16(outs, sizes, dest, n, bounds)
    torch.cuda.synchronize()
    got = bits_of(dest).reshape(count, n)
    for i in range(count):
        ref_out = np.zeros(n, dtype=np.uint16)
        co.decode(outs[i][: sizes[i]].cpu().numpy(), n, bounds[i], out_bf16=ref_out)
        assert bf16_equal(got[i], ref_out)
        x = host[i].float().numpy()
        xh = dest[i * n:(i + 1) * n].float().cpu().numpy()
        tol = bounds[i] * 1.01 + 1e-7 + np.abs(x) * 2.0 ** -8
        assert np.all(np.abs(x - xh) <= tol)


def test_random_sizes_match_oracle(cpp, co):
    rng = np.random.default_rng(7)
    w = make_wrapper(cpp, 1e-4)
    for trial in range(12):
        n = int(rng.integers(1, 300000))
        count = int(rng.integers(1, 4))
        eb = float(10.0 ** rng.uniform(-6, -2))
        host = _kv_pages(((n + 127) // 128) * 128, count, seed=trial)[:, :n].contiguous()
        bits = host.view(torch.int16).numpy().view(np.uint16)
        pages = [host[i].cuda() for i in range(count)]
        cap = max(int(w.estimate_compressed_buffer_size(n * 4)), 2048 + 132 * (n // 32 + 1))
        outs = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in pages]
        ok, sizes, bounds = w.compress_batch_fixed_bf16(pages, outs, [eb] * count)
        assert ok, n
        for i in range(count):
            ref, ref_eb = co.encode(bits[i], eb, relative=True)
            assert sizes[i] == ref.size, (n, i)
            assert np.array_equal(outs[i][: sizes[i]].cpu().numpy(), ref), (n, i)


def test_full_size_round_trip_properties(cpp):
    """The bench workload (256 Qwen2.5-1.5B pages, REL 1e-5): every element
    within bound; encoding is deterministic."""
    n, count, eb = 229376, 256, 1e-5
    host = _kv_pages(n, count, seed=0)
    pages = host.cuda()
    w = make_wrapper(cpp, eb)
    cap = int(w.estimate_compressed_buffer_size(n * 4))
    slab = torch.empty(count * cap, dtype=torch.uint8, device="cuda")
    outs = [slab[i * cap:(i + 1) * cap] for i in range(count)]
    ok, sizes, bounds = w.compress_batch_fixed_bf16(list(pages), outs, [eb] * count)
    assert ok
    dest = torch.zeros_like(pages)
    assert w.decompress_batch_fixed_bf16(outs, sizes, dest.view(-1), n, bounds)
    torch.cuda.synchronize()
    x, xh = pages.float(), dest.float()
    b = torch.tensor(bounds, device="cuda").view(-1, 1)
    assert bool(((x - xh).abs() <= b * 1.01 + 1e-7 + x.abs() * 2.0 ** -8).all())
    # deterministic: a second encode of the same pages gives the same bytes
    slab2 = torch.empty_like(slab)
    outs2 = [slab2[i * cap:(i + 1) * cap] for i in range(count)]
    ok, sizes2, bounds2 = w.compress_batch_fixed_bf16(list(pages), outs2, [eb] * count)
    assert ok and sizes2 == sizes and bounds2 == bounds
    for i in range(0, count, 37):
        assert torch.equal(outs[i][: sizes[i]], outs2[i][: sizes[i]])


def test_fp32_paths(cpp, co):
    """compress / decompress / compress_batch_fixed / decompress_batch use the
    same fixed-mode layout for FP32 input (upstream cuSZp's FP32 kernels,
    cuszp_fastpath.cu:5-64, are not vendored by the reference)."""
    w = make_wrapper(cpp, 1e-5)
    g = torch.Generator().manual_seed(3)
    inputs = [torch.randn(65536, generator=g), torch.randn(65536, generator=g) * 3.0]
    dev = [t.cuda() for t in inputs]
    cap = int(w.estimate_compressed_buffer_size(65536 * 4))
    outs = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in dev]
    ok, sizes, bounds = w.compress_batch_fixed(dev, outs, [1e-5, 1e-5])
    assert ok
    for t, o, s, b in zip(inputs, outs, sizes, bounds):
        ref, ref_eb = co.encode(t.numpy(), 1e-5, relative=True)
        assert np.float32(b).tobytes() == np.float32(ref_eb).tobytes()
        assert np.array_equal(o[:s].cpu().numpy(), ref)
        restored = torch.empty(65536, dtype=torch.float32, device="cuda")
        assert w.decompress(o, s, restored, b)
        torch.cuda.synchronize()
        assert float((restored.cpu() - t).abs().max()) <= b * 1.01 + 1e-7
    ok, buf, size, eb = w.compress(dev[0], torch.empty(0, dtype=torch.uint8, device="cuda"))
    assert ok and size == sizes[0] and eb == bounds[0]
    restored = [torch.empty(65536, device="cuda") for _ in dev]
    assert w.decompress_batch(outs, sizes, restored, bounds)
    torch.cuda.synchronize()
    for t, r, b in zip(inputs, restored, bounds):
        assert float((r.cpu() - t).abs().max()) <= b * 1.01 + 1e-7


def test_bf16_stream_decodes_with_fp32_decoder(cpp):
    """The reference's own cross-layout check (tests/test_vllm_v1_compressed_
    offload.py:47-110): BF16 indexed encode, FP32 decode."""
    w = make_wrapper(cpp, 1e-5)
    prefix, layers, epl = 2, 8, 4096
    sel = torch.tensor([1, 3, 6], dtype=torch.long, device="cuda")
    g = torch.Generator().manual_seed(11)
    inputs = [torch.randn(prefix * layers * epl, generator=g).to(torch.bfloat16).cuda()
              for _ in range(2)]
    n = prefix * sel.numel() * epl
    cap = int(w.estimate_compressed_buffer_size(n * 4))
    outs = [torch.empty(cap, dtype=torch.uint8, device="cuda") for _ in inputs]
    ok, sizes, bounds = w.compress_batch_fixed_bf16_indexed(
        inputs, outs, sel, prefix, layers, epl, [1e-5] * 2)
    assert ok
    for src, o, s, b in zip(inputs, outs, sizes, bounds):
        expected = src.view(prefix, layers, epl).index_select(1, sel).reshape(-1)
        restored = torch.empty(n, dtype=torch.float32, device="cuda")
        assert w.decompress(o, s, restored, b)
        torch.cuda.synchronize()
        assert float((restored - expected.float()).abs().max()) <= b * 1.01 + 1e-7


def test_indexed_groups_one_launch(cpp, co):
    """Mixed per-layer bounds (21 layers at 1e-4, 7 at 1e-5, the reference's
    calibrated profile) encoded by one launch; every unit bit-exact."""
    layers, prefix, epl = 28, 2, 4096
    low = [0, 1, 2, 5, 19, 20, 21]
    high = [i for i in range(layers) if i not in low]
    pages = _kv_pages(prefix * layers * epl, 3, seed=5)
    bits = pages.view(torch.int16).numpy().view(np.uint16)
    dev = [p.cuda() for p in pages]
    w = make_wrapper(cpp, 1e-5)
    groups = [torch.tensor(high, device="cuda"), torch.tensor(low, device="cuda")]
    inputs = dev + dev
    caps = [int(w.estimate_compressed_buffer_size(prefix * len(g) * epl * 4)) for g in groups]
    outs = [torch.empty(caps[0], dtype=torch.uint8, device="cuda") for _ in dev] + \
           [torch.empty(caps[1], dtype=torch.uint8, device="cuda") for _ in dev]
    eps = [1e-4] * 3 + [1e-5] * 3
    before = cpp.kernel_launches()
    ok, sizes, bounds = w.compress_batch_fixed_bf16_indexed_groups(
        inputs, outs, groups, [3, 3], prefix, layers, epl, eps)
    # one encode kernel for all groups (and its descriptor fetch kernel)
    assert ok and cpp.kernel_launches() - before == 2
    for k in range(6):
        sel = high if k < 3 else low
        ref, ref_eb = co.encode(bits[k % 3], eps[k], relative=True, layer_indices=sel,
                                prefix_count=prefix, source_layers=layers,
                                elements_per_layer=epl)
        assert sizes[k] == ref.size and np.array_equal(outs[k][: sizes[k]].cpu().numpy(), ref)
    # restore both groups into zeroed pages, one launch per group
    dests = [torch.zeros_like(d) for d in dev]
    assert w.decompress_batch_fixed_bf16_indexed_scatter(
        outs[:3], sizes[:3], dests, groups[0], prefix, layers, epl, bounds[:3])
    assert w.decompress_batch_fixed_bf16_indexed_scatter(
        outs[3:], sizes[3:], dests, groups[1], prefix, layers, epl, bounds[3:])
    torch.cuda.synchronize()
    for d, src, i in zip(dests, dev, range(3)):
        err = (d.float() - src.float()).abs().view(prefix, layers, epl)
        assert float(err[:, high].max()) <= bounds[i] * 1.01 + 1e-7 + 2 ** -8 * float(src.float().abs().max())
        assert float(err[:, low].max()) <= bounds[3 + i] * 1.01 + 1e-7 + 2 ** -8 * float(src.float().abs().max())


def test_zero_fill_option(cpp):
    case, z, sentinel = golden("zero_runs")
    w = make_wrapper(cpp)
    w.set_zero_fill(True)
    streams = _golden_streams(case, z)
    out = torch.full((case.batch * case.n,), sentinel, dtype=torch.int16,
                     device="cuda").view(torch.bfloat16)
    assert w.decompress_batch_fixed_bf16(streams, [int(s) for s in z["sizes"]], out, case.n,
                                         [float(b) for b in z["bounds"]])
    torch.cuda.synchronize()
    got = bits_of(out).reshape(case.batch, case.n)
    ref = z["decoded"]
    untouched = ref == sentinel
    assert untouched.any()
    assert np.all(got[untouched] == 0)
    assert np.array_equal(got[~untouched], ref[~untouched])


def test_error_behaviour(cpp):
    w = make_wrapper(cpp)
    page = torch.randn(8192, device="cuda").to(torch.bfloat16)
    small = torch.empty(100, dtype=torch.uint8, device="cuda")
    good = torch.empty(8 * 8192, dtype=torch.uint8, device="cuda")
    assert w.compress_batch_fixed_bf16([page], [small], [1e-4])[0] is False
    assert w.compress_batch_fixed_bf16([], [], [])[0] is False
    assert w.compress_batch_fixed_bf16([page.float()], [good], [1e-4])[0] is False
    assert w.compress_batch_fixed_bf16([page.cpu()], [good], [1e-4])[0] is False
    assert w.compress_batch_fixed_bf16([page], [good], [1e-4, 1e-4])[0] is False
    plain = cpp.CuSZpWrapper(cpp.CompressionConfig(), 0)   # default mode: plain
    assert plain.compress_batch_fixed_bf16([page], [good], [1e-4])[0] is False
    ok, sizes, bounds = w.compress_batch_fixed_bf16([page], [good], [1e-4])
    assert ok
    out = torch.empty(8192, dtype=torch.bfloat16, device="cuda")
    assert w.decompress_batch_fixed_bf16([], [], out, 8192, []) is True
    assert w.decompress_batch_fixed_bf16([good], [0], out, 8192, bounds) is False
    # a truncated stream is reported, not read past its size
    assert w.decompress_batch_fixed_bf16([good], [sizes[0] - 4], out, 8192, bounds)
    assert w.device_status() & 4
    assert w.device_status() == 0
    # a size below the header (1024 rate bytes here) is refused before launch
    assert w.decompress_batch_fixed_bf16([good], [1020], out, 8192, bounds) is False
    # tiny units: the header alone exceeds 8 * n bytes -> capacity error
    tiny = torch.randn(16, device="cuda").to(torch.bfloat16)
    assert w.compress_batch_fixed_bf16([tiny], [torch.empty(128, dtype=torch.uint8,
                                                            device="cuda")], [])[0] is False


def test_units_above_the_encoder_limit_are_refused(cpp):
    """Units above 16 slices of 100 KB (819200 BF16 elements) are refused
    (False, no launch) rather than encoded wrongly."""
    n = 819201
    w = make_wrapper(cpp, 1e-4)
    page = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(int(w.estimate_compressed_buffer_size(n * 4)), dtype=torch.uint8,
                      device="cuda")
    before = cpp.kernel_launches()
    ok, _sizes, _bounds = w.compress_batch_fixed_bf16([page], [out], [1e-4])
    assert not ok and cpp.kernel_launches() == before
