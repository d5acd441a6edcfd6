"""The INT8 comparison codec's oracle (oracle/int8_codec.py) on CPU: known
answers, and agreement with the reference's torch expression of it
(vllm_v1_compressed_offload.py:711-724 and :2094-2097) run with CPU torch on
the same seeded pages.  On the reference's device (CUDA tensors) ATen turns
``max / 127.0`` into a multiply by the float32 reciprocal; CPU torch divides,
so the scale is formed here as the CUDA code path forms it.  The GPU tests
compare with CUDA torch itself."""
import numpy as np
import torch

from oracle import int8_codec as oc


def _bits(values):
    return torch.tensor(values, dtype=torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def test_known_answers():
    q, scale = oc.encode(_bits([1.0, -2.0, 0.5, 127.0, 2.5, -3.5, -127.0, 0.0]))
    assert scale == np.float32(1.0)
    # round half to even: 0.5 -> 0, 2.5 -> 2, -3.5 -> -4
    assert q.tolist() == [1, -2, 0, 127, 2, -4, -127, 0]
    assert oc.decode(q, scale).tolist() == _bits([1, -2, 0, 127, 2, -4, -127, 0]).tolist()


def test_zero_page_uses_unit_scale():
    q, scale = oc.encode(np.zeros(64, dtype=np.uint16))
    assert scale == np.float32(1.0) and not q.any()


def test_stored_layout():
    q, scale = oc.encode(_bits([3.0, -1.0, 2.0, 1.0, 5.0]))
    blob = oc.stored_page(q, scale)
    assert len(blob) == 8 + 4
    assert np.frombuffer(blob[:5], dtype=np.int8).tolist() == q.tolist()
    assert np.frombuffer(blob[8:], dtype=np.float32)[0] == scale


def test_matches_reference_expression_on_cpu_torch():
    g = torch.Generator().manual_seed(7)
    for n, spread in [(4096, 1.0), (36864, 0.05), (1000, 40.0)]:
        page = (torch.randn(n, generator=g) * spread).to(torch.bfloat16)
        # the reference's store and restore, verbatim in meaning
        x = page.to(torch.float32)
        scale_t = x.abs().max() * torch.tensor(1.0 / 127.0, dtype=torch.float32)
        if float(scale_t.item()) == 0.0:
            scale_t = torch.ones_like(scale_t)
        ref_q = torch.clamp(torch.round(x / scale_t), -127, 127).to(torch.int8)
        ref_out = (ref_q.to(torch.float32) * float(scale_t.item())).to(torch.bfloat16)
        q, scale = oc.encode(page.view(torch.int16).numpy().view(np.uint16))
        assert scale == np.float32(scale_t.item())
        assert np.array_equal(q, ref_q.numpy())
        assert np.array_equal(oc.decode(q, scale), ref_out.view(torch.int16).numpy().view(np.uint16))
