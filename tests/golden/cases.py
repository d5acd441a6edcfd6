"""Seeded golden cases for the fixed-mode codec (test infrastructure).

Each case is a batch of BF16 units with one shape and one requested bound.
Inputs are generated here from fixed seeds; make_golden.py runs the
reference's own kernels on them (on a B200) and stores the outputs.  The
tests regenerate the inputs, check them against the stored SHA-256 of the
input bits, and compare every implementation with the stored outputs.

The distributions follow the workloads the reference measures (KV pages of
[2 (K/V), layers, heads, 16 tokens, head_dim] BF16 values, per-channel
LogNormal scales, a few outlier channels), scaled down, plus edge cases:
ragged sizes around the 32-element block and 32768-element group
boundaries, runs of zeros (rate-0 blocks), constant pages, NaN/Inf/zero/
subnormal specials, and values picked so that a fused multiply-add in the
quantiser gives a different integer than separate multiply and add.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

HEAD_DIM = 128


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


@dataclass
class Case:
    name: str
    n: int                      # logical elements per unit
    batch: int
    eps: float                  # requested bound per unit
    relative: bool = True
    kind: str = "kv"
    seed: int = 0
    # layer-indexed units: source page [prefix][source_layers][epl]
    layer_indices: tuple[int, ...] | None = None
    prefix_count: int = 0
    source_layers: int = 0
    elements_per_layer: int = 0
    # decode destinations split per unit (scatter mode) when > 1
    destinations_per_page: int = 1
    # per-unit requested bounds, overriding eps
    unit_eps: tuple[float, ...] | None = None
    extra: dict = field(default_factory=dict)

    def eps_of(self, unit: int) -> float:
        return self.unit_eps[unit] if self.unit_eps else self.eps

    @property
    def source_numel(self) -> int:
        if self.layer_indices is None:
            return self.n
        return self.prefix_count * self.source_layers * self.elements_per_layer


def _kv_values(rng: np.random.Generator, numel: int) -> np.ndarray:
    """K-like values: N(0,1) times a per-channel LogNormal(0, 0.5) scale,
    with 4 outlier channels scaled by 8 (head_dim channels innermost)."""
    channels = HEAD_DIM
    scale = rng.lognormal(0.0, 0.5, channels).astype(np.float32)
    scale[rng.choice(channels, 4, replace=False)] *= 8.0
    x = rng.standard_normal(numel).astype(np.float32)
    reps = (numel + channels - 1) // channels
    return x * np.tile(scale, reps)[:numel]


# (value, absolute bound) pairs where x * (0.5 / bound), rounded to FP32,
# lands exactly on -(2**k + 0.5) although the exact product does not: there
# the separately rounded add gives -2**k and the fused one gives a value
# just above it, so the two quantiser forms differ by one.
FMA_PROBES = (
    (-0.240234375, 0.080078125),
    (-0.369140625, 0.0014363449299708009),
    (-0.07470703125, 7.288491178769618e-05),
)


def _fma_probe(rng: np.random.Generator, numel: int, unit: int) -> np.ndarray:
    x0, eb = FMA_PROBES[unit % len(FMA_PROBES)]
    out = (rng.standard_normal(numel) * 200.0 * eb).astype(np.float32)
    pos = rng.choice(numel, numel // 8, replace=False)
    out[pos] = np.float32(x0)
    return out


def _specials(rng: np.random.Generator, numel: int) -> np.ndarray:
    x = rng.standard_normal(numel).astype(np.float32)
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-40,
                         3.0e38, -3.0e38, 65504.0], dtype=np.float32)
    pos = rng.choice(numel, min(numel, 40), replace=False)
    x[pos] = specials[np.arange(pos.size) % specials.size]
    return x


def unit_values(case: Case, unit: int) -> np.ndarray:
    """FP32 values of one source page (before BF16 rounding)."""
    rng = np.random.default_rng([case.seed, unit])
    numel = case.source_numel
    if case.kind == "kv":
        return _kv_values(rng, numel)
    if case.kind == "gauss":
        return rng.standard_normal(numel).astype(np.float32)
    if case.kind == "zero_runs":
        x = _kv_values(rng, numel)
        mask = (np.arange(numel) // 96) % 3 == 1
        x[mask] = 0.0
        return x
    if case.kind == "tiny_runs":
        # blocks whose values all quantise to zero without being zero
        x = _kv_values(rng, numel)
        mask = (np.arange(numel) // 64) % 4 == 2
        x[mask] *= 1e-7
        return x
    if case.kind == "const":
        return np.full(numel, 1.5, dtype=np.float32)
    if case.kind == "specials":
        return _specials(rng, numel)
    if case.kind == "specials_finite":
        x = _specials(rng, numel)
        x[~np.isfinite(x) & ~np.isnan(x)] = 2.0
        x[np.abs(x) > 1e30] = -3.0
        return x
    if case.kind == "fma_probe":
        return _fma_probe(rng, numel, unit)
    raise ValueError(case.kind)


def unit_bits(case: Case, unit: int) -> np.ndarray:
    return f32_to_bf16_bits(unit_values(case, unit))


def inputs_sha256(case: Case) -> str:
    h = hashlib.sha256()
    for u in range(case.batch):
        h.update(unit_bits(case, u).tobytes())
    return h.hexdigest()


CASES: list[Case] = [
    Case("n1", 1, 2, 1e-4, seed=1),
    Case("n31", 31, 2, 1e-4, seed=2),
    Case("n32", 32, 2, 1e-4, seed=3),
    Case("n33", 33, 2, 1e-4, seed=4),
    Case("n1000_odd", 1001, 2, 1e-3, seed=5, kind="gauss"),
    Case("c1_unit", 8192, 4, 1e-4, seed=6),
    Case("n32767", 32767, 1, 1e-5, seed=7),
    Case("n32768", 32768, 1, 1e-5, seed=8),
    Case("n32769", 32769, 1, 1e-5, seed=9),
    Case("min_cuszp", 36864, 2, 1e-5, seed=10),
    Case("three_groups", 65636, 1, 1e-4, seed=11),
    Case("abs_bound", 4096, 2, 2e-3, relative=False, seed=12, kind="gauss"),
    Case("zero_runs", 8192, 2, 1e-4, seed=13, kind="zero_runs"),
    Case("tiny_runs", 8192, 2, 1e-3, seed=14, kind="tiny_runs"),
    Case("const", 4096, 2, 1e-5, seed=15, kind="const"),
    Case("specials", 2048, 2, 1e-3, seed=16, kind="specials"),
    Case("specials_finite", 2048, 2, 1e-3, seed=23, kind="specials_finite"),
    Case("fma_probe", 4096, 3, 0.0, relative=False, seed=17, kind="fma_probe",
         unit_eps=tuple(eb for _x0, eb in FMA_PROBES)),
    Case("scatter2", 8192, 3, 1e-4, seed=19, destinations_per_page=2),
    Case("scatter4", 12288, 2, 1e-5, seed=20, destinations_per_page=4),
    Case("indexed", 2 * 3 * 4096, 2, 1e-5, seed=21,
         layer_indices=(1, 3, 6), prefix_count=2, source_layers=8,
         elements_per_layer=4096),
    Case("indexed_ragged", 2 * 2 * 1000, 2, 1e-4, seed=22,
         layer_indices=(4, 0), prefix_count=2, source_layers=5,
         elements_per_layer=1000),
]

CASE_BY_NAME = {c.name: c for c in CASES}
