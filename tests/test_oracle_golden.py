"""The CPU oracle against the golden vectors from the reference's kernels.

tests/golden/fixtures holds, per case in tests/golden/cases.py, the output of
the reference's own integration/cuszp_wrapper/cuszp_batched_fixed.cu kernels
run on a B200 (tests/golden/make_golden.py).  These tests pin the C oracle
(oracle/fixed_codec.c) to them: compressed bytes, sizes and resolved bounds
byte-identical, decoded BF16 bit-identical (NaN compared as NaN), with the
quantiser in its separately rounded multiply-then-add form -- the fused
form is shown NOT to reproduce the reference on the probe case.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from cases import CASES, CASE_BY_NAME, inputs_sha256, unit_bits
from oracle.oracle import COracle, np_decode, np_encode, bf16_bits_to_f32

FIX = Path(__file__).resolve().parent / "golden" / "fixtures"
MANIFEST = json.loads((FIX / "manifest.json").read_text())
SENTINEL = MANIFEST["sentinel"]


@pytest.fixture(scope="module")
def co():
    return COracle()


def _layer_kw(case):
    if case.layer_indices is None:
        return {}
    return dict(layer_indices=case.layer_indices, prefix_count=case.prefix_count,
                source_layers=case.source_layers,
                elements_per_layer=case.elements_per_layer)


def _units(case):
    z = np.load(FIX / f"{case.name}.npz")
    off = 0
    out = []
    for u in range(case.batch):
        size = int(z["sizes"][u])
        out.append((z["compressed"][off:off + size], float(z["bounds"][u])))
        off += size
    return z, out


def _bf16_equal(a, b):
    na = (a & 0x7FFF) > 0x7F80
    nb = (b & 0x7FFF) > 0x7F80
    return np.array_equal(na, nb) and np.array_equal(a[~na], b[~nb])


@pytest.mark.parametrize("name", [c.name for c in CASES])
def test_inputs_regenerate(name):
    case = CASE_BY_NAME[name]
    assert inputs_sha256(case) == MANIFEST["cases"][name]["inputs_sha256"]


@pytest.mark.parametrize("name", [c.name for c in CASES])
def test_oracle_encode_matches_reference_kernels(co, name):
    case = CASE_BY_NAME[name]
    z, units = _units(case)
    for u, (ref_bytes, ref_eb) in enumerate(units):
        buf, eb = co.encode(unit_bits(case, u), case.eps_of(u),
                            relative=case.relative, fused=False, **_layer_kw(case))
        assert np.float32(eb).tobytes() == np.float32(ref_eb).tobytes()
        assert buf.size == ref_bytes.size
        assert np.array_equal(buf, ref_bytes)


@pytest.mark.parametrize("name", [c.name for c in CASES])
def test_oracle_decode_matches_reference_kernels(co, name):
    case = CASE_BY_NAME[name]
    z, units = _units(case)
    for u, (ref_bytes, ref_eb) in enumerate(units):
        kw = _layer_kw(case)
        kw.pop("prefix_count", None)
        out = np.full(case.source_numel, SENTINEL, dtype=np.uint16)
        co.decode(ref_bytes, case.n, ref_eb, out_bf16=out, **kw)
        assert _bf16_equal(out, z["decoded"][u])


def test_fused_quantiser_does_not_reproduce_reference(co):
    """The probe case separates the two quantiser forms; only the separately
    rounded one matches the reference's kernels."""
    case = CASE_BY_NAME["fma_probe"]
    assert MANIFEST["cases"]["fma_probe"]["oracle_match"] == {
        "separate": True, "fused": False}
    _, units = _units(case)
    mismatched = 0
    for u, (ref_bytes, _eb) in enumerate(units):
        buf, _ = co.encode(unit_bits(case, u), case.eps_of(u),
                           relative=False, fused=True)
        mismatched += int(buf.size != ref_bytes.size
                          or not np.array_equal(buf, ref_bytes))
    assert mismatched == case.batch


@pytest.mark.parametrize("name", ["n33", "n1000_odd", "c1_unit", "zero_runs",
                                  "specials_finite", "fma_probe", "abs_bound"])
def test_numpy_restatement_agrees(name):
    """A second, independent restatement (numpy) gives the same bytes."""
    case = CASE_BY_NAME[name]
    z, units = _units(case)
    for u, (ref_bytes, ref_eb) in enumerate(units):
        vals = bf16_bits_to_f32(unit_bits(case, u))
        assert np.array_equal(np_encode(vals, ref_eb, fused=False), ref_bytes)
        dec, written = np_decode(ref_bytes, case.n, ref_eb)
        golden = bf16_bits_to_f32(z["decoded"][u])
        assert np.array_equal(np.isnan(dec[written]), np.isnan(golden[written]))
        fin = written & ~np.isnan(dec)
        from oracle.oracle import f32_to_bf16_bits
        assert np.array_equal(f32_to_bf16_bits(dec[fin]), z["decoded"][u][fin])
        # blocks the reference decoder does not write keep the sentinel
        assert np.all(z["decoded"][u][~written] == SENTINEL)


@pytest.mark.parametrize("name", ["c1_unit", "min_cuszp", "indexed", "scatter4"])
def test_error_bound(co, name):
    """|x - x_hat_bf16| <= eb*1.01 + 1e-7 + one BF16 ulp of x (the reference's
    test tolerance, tests/test_vllm_v1_compressed_offload.py:884-889)."""
    case = CASE_BY_NAME[name]
    z, units = _units(case)
    for u, (ref_bytes, eb) in enumerate(units):
        bits = unit_bits(case, u)
        x = bf16_bits_to_f32(bits)
        xh = bf16_bits_to_f32(z["decoded"][u])
        if case.layer_indices is not None:
            view = np.arange(case.source_numel).reshape(
                case.prefix_count, case.source_layers, case.elements_per_layer)
            sel = view[:, list(case.layer_indices), :].reshape(-1)
            x, xh = x[sel], xh[sel]
        tol = eb * 1.01 + 1e-7 + np.abs(x) * 2.0 ** -8
        assert np.all(np.abs(x - xh) <= tol)
