"""Python access to the test oracles (test infrastructure only).

Two independent CPU restatements of the reference's fixed-mode codec
(integration/cuszp_wrapper/cuszp_batched_fixed.cu):

* :class:`COracle` -- ctypes bindings to ``fixed_codec.c`` (fast; used by
  the parity tests, the smoke check and bench.py's CPU baseline);
* ``np_*`` functions -- a vectorised numpy restatement written separately,
  used only on small inputs to cross-check the C one.

And :class:`RefKernels` -- ctypes bindings to the reference's own CUDA
kernels built into ``oracle/_ref`` (GPU box only), used to generate and
re-check the golden bitstreams.

Nothing here is imported by the product package.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import build as _build

GROUP = 32768
BLOCK = 32

c_size = C.c_size_t
c_float = C.c_float
c_int = C.c_int
c_void_p = C.c_void_p


def header_bytes(n: int) -> int:
    return (n + GROUP - 1) // GROUP * (GROUP // BLOCK)


def capacity_for(n: int) -> int:
    """Worst-case compressed bytes for n elements (every block at rate 31)."""
    nblocks = (n + BLOCK - 1) // BLOCK
    return header_bytes(n) + nblocks * (4 + 4 * 32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round to nearest even; NaN -> 0x7FFF (as __float2bfloat16_rn)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


class COracle:
    """ctypes view of oracle/fixed_codec.c."""

    def __init__(self, path: Path | None = None):
        self.path = Path(path) if path else _build.build_oracle()
        lib = C.CDLL(str(self.path))
        lib.ckvo_quantize.restype = C.c_int32
        lib.ckvo_quantize.argtypes = [c_float, c_float, c_int]
        lib.ckvo_relative_bound.restype = c_float
        lib.ckvo_relative_bound.argtypes = [
            c_void_p, c_int, c_size, c_float, c_void_p, c_size, c_size, c_size]
        lib.ckvo_encode.restype = c_size
        lib.ckvo_encode.argtypes = [
            c_void_p, c_int, c_size, c_float, c_int, c_void_p, c_size, c_size,
            c_size, c_void_p, c_size, c_int, C.POINTER(c_float)]
        lib.ckvo_decode.restype = c_size
        lib.ckvo_decode.argtypes = [
            c_void_p, c_size, c_size, c_float, c_void_p, c_void_p, c_void_p,
            c_size, c_size, c_size, c_int]
        lib.ckvo_f32_to_bf16.restype = C.c_uint16
        lib.ckvo_f32_to_bf16.argtypes = [c_float]
        lib.ckvo_encode_batch_bf16.restype = c_int
        lib.ckvo_encode_batch_bf16.argtypes = [
            c_void_p, c_void_p, c_size, c_size, c_size, c_float, c_int, c_int,
            c_void_p, c_void_p, c_int]
        lib.ckvo_decode_batch_bf16.restype = c_int
        lib.ckvo_decode_batch_bf16.argtypes = [
            c_void_p, c_void_p, c_void_p, c_void_p, c_size, c_size, c_int]
        self.lib = lib

    @staticmethod
    def _layers(layer_indices, selected_layers, source_layers, elements_per_layer):
        if layer_indices is None:
            return None, 0, 0, 0, None
        idx = np.ascontiguousarray(layer_indices, dtype=np.int64)
        return idx.ctypes.data, len(idx), source_layers, elements_per_layer, idx

    def quantize(self, x: float, recip: float, fused: bool) -> int:
        return int(self.lib.ckvo_quantize(x, recip, int(fused)))

    def relative_bound(self, data: np.ndarray, eb: float, n: int | None = None,
                       layer_indices=None, source_layers=0,
                       elements_per_layer=0) -> float:
        is_bf16 = data.dtype == np.uint16
        data = np.ascontiguousarray(data)
        ptr, sel, src, epl, keep = self._layers(
            layer_indices, 0, source_layers, elements_per_layer)
        if n is None:
            n = data.size if layer_indices is None else 0
        return float(self.lib.ckvo_relative_bound(
            data.ctypes.data, int(is_bf16), n, eb, ptr, sel, src, epl))

    def encode(self, data: np.ndarray, eb: float, *, relative: bool = True,
               fused: bool = False, n: int | None = None, layer_indices=None,
               prefix_count: int = 0, source_layers: int = 0,
               elements_per_layer: int = 0) -> tuple[np.ndarray, float]:
        """Encode one unit; data is uint16 (BF16 bits) or float32.

        Returns (compressed bytes, resolved absolute bound).
        """
        is_bf16 = data.dtype == np.uint16
        data = np.ascontiguousarray(data)
        ptr, sel, src, epl, keep = self._layers(
            layer_indices, 0, source_layers, elements_per_layer)
        if n is None:
            n = data.size if layer_indices is None else prefix_count * sel * epl
        cap = capacity_for(n)
        out = np.zeros(cap, dtype=np.uint8)
        eb_out = c_float(0.0)
        size = self.lib.ckvo_encode(
            data.ctypes.data, int(is_bf16), n, eb, int(relative), ptr, sel, src,
            epl, out.ctypes.data, cap, int(fused), C.byref(eb_out))
        if size == 0:
            raise RuntimeError("oracle encode overflowed its buffer")
        return out[:size].copy(), float(eb_out.value)

    def decode(self, buf: np.ndarray, n: int, eb: float, *, out_bf16=None,
               out_f32=None, layer_indices=None, source_layers=0,
               elements_per_layer=0, write_zero_blocks: bool = False) -> int:
        """Decode into caller arrays (prefilled; rate-0 blocks are skipped)."""
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        ptr, sel, src, epl, keep = self._layers(
            layer_indices, 0, source_layers, elements_per_layer)
        consumed = self.lib.ckvo_decode(
            buf.ctypes.data, buf.size, n, eb,
            out_f32.ctypes.data if out_f32 is not None else None,
            out_bf16.ctypes.data if out_bf16 is not None else None,
            ptr, sel, src, epl, int(write_zero_blocks))
        if consumed == C.c_size_t(-1).value:
            raise ValueError("oracle decode found an invalid bitstream")
        return int(consumed)

    def encode_batch_bf16(self, pages: list[np.ndarray], eb: float, *,
                          relative=True, fused=False, threads=1):
        n = pages[0].size
        cap = capacity_for(n)
        outs = [np.zeros(cap, dtype=np.uint8) for _ in pages]
        pp = (c_void_p * len(pages))(*[p.ctypes.data for p in pages])
        op = (c_void_p * len(pages))(*[o.ctypes.data for o in outs])
        sizes = np.zeros(len(pages), dtype=np.uint64)
        ebs = np.zeros(len(pages), dtype=np.float32)
        rc = self.lib.ckvo_encode_batch_bf16(
            pp, op, len(pages), n, cap, eb, int(relative), int(fused),
            sizes.ctypes.data, ebs.ctypes.data, threads)
        if rc != 0:
            raise RuntimeError("oracle batch encode failed")
        return outs, sizes, ebs


# ---------------------------------------------------------------------------
# Independent numpy restatement (small inputs only).


def np_quantize(x: np.ndarray, recip: np.float32, fused: bool) -> np.ndarray:
    """batch_quantization (cuszp_batched_fixed.cu:10-25), elementwise."""
    x = np.asarray(x, dtype=np.float32)
    recip = np.float32(recip)
    with np.errstate(all="ignore"):
        r = (x * recip).astype(np.float32)
        s = np.where(r >= np.float32(-0.5), 0, 1).astype(np.int64)
        if fused:
            # x*recip is exact in float64 for BF16/FP32 inputs; adding 0.5 is
            # exact wherever the truncated result can depend on it.
            t = (x.astype(np.float64) * np.float64(recip) + 0.5).astype(np.float32)
        else:
            t = (r + np.float32(0.5)).astype(np.float32)
        c = np.zeros(t.shape, dtype=np.int64)
        finite = ~np.isnan(t)
        tt = t[finite].astype(np.float64)
        c[finite] = np.clip(np.trunc(tt), -2**31, 2**31 - 1).astype(np.int64)
    q = c - s
    q = ((q + 2**31) % 2**32) - 2**31  # sub.s32 wraps
    return q.astype(np.int64)


def np_encode(values_f32: np.ndarray, eb_abs: float, fused: bool) -> np.ndarray:
    """Encode logical FP32 values (cuszp_batched_fixed.cu:135-359)."""
    n = values_f32.size
    hdr = header_bytes(n)
    nblocks = (n + BLOCK - 1) // BLOCK
    recip = np.float32(np.float32(0.5) / np.float32(eb_abs))
    q = np.zeros(nblocks * BLOCK, dtype=np.int64)
    q[:n] = np_quantize(values_f32, recip, fused)
    q = q.reshape(nblocks, BLOCK)
    neg = q < 0
    a = np.where(neg, -q, q).astype(np.uint64)
    rates = np.array([int(v).bit_length() for v in a.max(axis=1)], dtype=np.uint8)
    out = bytearray(hdr)
    out[:nblocks] = rates.tobytes()
    weights = (1 << (31 - np.arange(32, dtype=np.uint64))).astype(np.uint64)
    for j in range(nblocks):
        r = int(rates[j])
        if not r:
            continue
        sign = int((neg[j].astype(np.uint64) * weights).sum())
        out += sign.to_bytes(4, "big")
        for b in range(r):
            plane = int((((a[j] >> np.uint64(b)) & np.uint64(1)) * weights).sum())
            out += plane.to_bytes(4, "big")
    return np.frombuffer(bytes(out), dtype=np.uint8)


def np_decode(buf: np.ndarray, n: int, eb: float) -> tuple[np.ndarray, np.ndarray]:
    """Decode to (FP32 values, written mask); rate-0 blocks are not written."""
    hdr = header_bytes(n)
    nblocks = (n + BLOCK - 1) // BLOCK
    out = np.zeros(nblocks * BLOCK, dtype=np.float32)
    written = np.zeros(nblocks * BLOCK, dtype=bool)
    off = hdr
    eb = np.float32(eb)
    for j in range(nblocks):
        r = int(buf[j])
        if not r:
            continue
        sign = int.from_bytes(bytes(buf[off:off + 4]), "big")
        off += 4
        a = np.zeros(BLOCK, dtype=np.int64)
        for b in range(r):
            plane = int.from_bytes(bytes(buf[off:off + 4]), "big")
            off += 4
            bits = (plane >> (31 - np.arange(32))) & 1
            a |= bits.astype(np.int64) << b
        negs = (sign >> (31 - np.arange(32))) & 1
        q = np.where(negs == 1, -a, a)
        with np.errstate(all="ignore"):
            v = (q.astype(np.float32) * eb).astype(np.float32) * np.float32(2.0)
        out[j * BLOCK:(j + 1) * BLOCK] = v
        written[j * BLOCK:(j + 1) * BLOCK] = True
    return out[:n], written[:n]


# ---------------------------------------------------------------------------
# The reference's own kernels (GPU only).


class RefKernels:
    """ctypes view of oracle/_ref/libref_fixed.so (the reference kernels)."""

    def __init__(self, path: Path | None = None):
        so = Path(path) if path else _build.REF_SO
        if not so.exists():
            raise FileNotFoundError(f"reference kernels not built: {so}")
        lib = C.CDLL(str(so))
        lib.ref_compress_bf16.restype = c_int
        lib.ref_compress_bf16.argtypes = [
            c_void_p, c_void_p, c_size, c_size, c_size, c_void_p, c_int,
            c_void_p, c_size, c_size, c_size, c_size, c_void_p, c_void_p,
            c_void_p, c_int]
        lib.ref_decompress_bf16.restype = c_int
        lib.ref_decompress_bf16.argtypes = [
            c_void_p, c_size, c_size, c_void_p, c_int, c_void_p, c_size, c_size,
            c_void_p, c_size, c_size, c_size, c_size, c_void_p]
        self.lib = lib

    def compress(self, input_ptrs, output_ptrs, capacity, n, eps, relative=True,
                 layer_indices_ptr=None, selected=0, prefix_count=0,
                 source_layers=0, elements_per_layer=0, stream=0,
                 zero_outputs=True):
        batch = len(input_ptrs)
        ip = (c_void_p * batch)(*input_ptrs)
        op = (c_void_p * batch)(*output_ptrs)
        e = np.ascontiguousarray(eps, dtype=np.float32)
        sizes = np.zeros(batch, dtype=np.uint64)
        bounds = np.zeros(batch, dtype=np.float32)
        rc = self.lib.ref_compress_bf16(
            ip, op, capacity, batch, n, e.ctypes.data, int(relative),
            layer_indices_ptr, selected, prefix_count, source_layers,
            elements_per_layer, sizes.ctypes.data, bounds.ctypes.data, stream,
            int(zero_outputs))
        if rc != 0:
            raise RuntimeError(f"reference compress failed ({rc})")
        return sizes, bounds

    def decompress(self, input_ptrs, n, bounds, mode, dest_ptrs, per_page=0,
                   elements_per_dest=0, layer_indices_ptr=None, selected=0,
                   prefix_count=0, source_layers=0, elements_per_layer=0,
                   stream=0):
        batch = len(input_ptrs)
        ip = (c_void_p * batch)(*input_ptrs)
        dp = (c_void_p * len(dest_ptrs))(*dest_ptrs)
        b = np.ascontiguousarray(bounds, dtype=np.float32)
        rc = self.lib.ref_decompress_bf16(
            ip, batch, n, b.ctypes.data, mode, dp, per_page, elements_per_dest,
            layer_indices_ptr, selected, prefix_count, source_layers,
            elements_per_layer, stream)
        if rc != 0:
            raise RuntimeError(f"reference decompress failed ({rc})")
