"""INT8 page codec of the reference's comparison protocol, restated in numpy
(test infrastructure only; never imported by the product package).

Follows integration/compression_pipeline/vllm_v1_compressed_offload.py:
  * :711-724 (store): ``scale = page.abs().max() / 127.0`` (1.0 when that is
    zero), ``q = clamp(round(page / scale), -127, 127).to(int8)``; the stored
    size is numel + 4 (the scale travels with the payload);
  * the page is a CUDA tensor there, and ATen divides a CUDA tensor by a CPU
    scalar as a multiply by the float32 reciprocal (BinaryDivTrueKernel.cu,
    "may lose one bit of precision"): scale = max|x| * RN(1/127); the page
    division ``page / scale`` (tensor by tensor) is a true division;
  * :2090-2116 (restore): ``q.to(float32) * scale``, then ``.to(bfloat16)``.
The page is the BF16 page widened to float32 (exact).  torch.round rounds
half to even, as np.rint does; the divisions and the multiply are float32
operations rounded to nearest, as numpy performs them on float32 operands.

The stored form used by the pipeline (ckv_pipe_store_int8) is the n int8
values followed by the float32 scale at byte align4(n).
"""
from __future__ import annotations

import numpy as np

from .oracle import bf16_bits_to_f32, f32_to_bf16_bits


def align4(n: int) -> int:
    return (n + 3) & ~3


def encode(page_bits: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """(int8 values, scale) of one page given as BF16 bit patterns."""
    x = bf16_bits_to_f32(np.ascontiguousarray(page_bits, dtype=np.uint16))
    with np.errstate(invalid="ignore", divide="ignore"):
        scale = np.float32(np.abs(x).max()) * (np.float32(1.0) / np.float32(127.0))
        if scale == np.float32(0.0):
            scale = np.float32(1.0)
        v = np.rint(x / scale)
        # clamp keeps NaN; the int8 cast on the GPU turns it into 0
        q = np.where(np.isnan(v), 0, np.clip(v, -127, 127)).astype(np.int8)
    return q, np.float32(scale)


def decode(q: np.ndarray, scale: np.float32) -> np.ndarray:
    """BF16 bit patterns restored from int8 values and their scale."""
    x = q.astype(np.float32) * np.float32(scale)
    return f32_to_bf16_bits(x.astype(np.float32))


def stored_page(q: np.ndarray, scale: np.float32) -> bytes:
    """The pipeline's stored bytes of one page."""
    n = q.size
    out = bytearray(align4(n) + 4)
    out[:n] = q.view(np.uint8).tobytes()
    out[align4(n):] = np.float32(scale).tobytes()
    return bytes(out)
