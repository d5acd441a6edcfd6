"""Compressed KV-page offload jobs: GPU blocks -> page-locked host memory -> GPU blocks.

The job layer of the reference's vLLM connector
(integration/compression_pipeline/vllm_v1_compressed_offload.py), for its
fixed-mode BF16 path, on top of libckv's store / restore pipeline
(``ckv_pipe_*``):

* ``BundleComponent`` / ``EncodedSegment`` / ``CompressedBundle`` -- the
  reference's per-page host metadata (:58-88), same fields;
* ``CompressedPageStore`` -- host storage shared by both directions
  (:360-457).  The reference packs each store job with ``torch.cat`` into a
  freshly allocated pinned slab and synchronises; here a job is written by
  the pipeline into a pinned slab taken from a reusable pool, and the slab
  starts with a self-describing header and page table (``JobHeader``), so a
  stored job can be validated and restored from its bytes alone;
* ``CompressedOffloadingHandler`` -- ``transfer_async`` / ``get_finished`` /
  ``wait`` / ``shutdown`` (:2365-2410) over vLLM-style specs (anything with a
  ``block_ids`` array, e.g. ``GPULoadStoreSpec`` / ``CPULoadStoreSpec``);
  page addresses come from the block ids in one vector operation (no
  per-page Python, the reference's ``_compress_fixed_bundles_batched`` loops
  over pages, :825-1028);
* ``CompressedCpuGpuOffloadingHandlers`` -- the pair of handlers (:2412-2470),
  sharing one store and one pipeline, so that a load is ordered after the
  store that wrote its pages on the device.

A KV cache here is one contiguous tensor ``[num_blocks, *page_shape]`` of
BF16 pages (the cross-layer page layout the reference compresses as one
unit, e.g. ``[2, layers, heads, 16, head_dim]``), or its byte storage.

What a stored page becomes follows the reference's handler: one cuSZp
fixed-mode stream per page, or with per-layer bounds one segment per
distinct bound (zero-bound layers raw); a page or segment that cuSZp would
not shrink below its BF16 size is stored raw; pages below 36864 elements are
coded zero-padded; and the handler's ``codec`` may instead be the
reference's ``"int8"`` or ``"raw"`` comparison codecs.
"""
from __future__ import annotations

import ctypes as C
import struct
import threading
from dataclasses import dataclass, field
from typing import Any, Iterable, Sequence

import numpy as np
import torch

import _ckv

# Smallest unit the reference's connector compresses; smaller pages are
# zero-padded to it (vllm_v1_compressed_offload.py:49).
MIN_CUSZP_ELEMENTS = 36864

# --------------------------------------------------------------------------
# Host metadata (vllm_v1_compressed_offload.py:58-88)


@dataclass
class BundleComponent:
    tensor_idx: int
    original_shape: tuple[int, ...]
    original_dtype: torch.dtype
    numel: int
    layer_axis: int | None = None
    layer_indices: tuple[int, ...] = ()
    destination_view_shape: tuple[int, ...] = ()


@dataclass
class EncodedSegment:
    payload: torch.Tensor            # view of the job's pinned slab
    compressed_size: int
    actual_error_bound: float
    encoding: str
    components: tuple[BundleComponent, ...]
    unpadded_numel: int
    compressed_numel: int
    original_bytes: int
    requested_error_bound: float
    quant_scale: float | None = None
    cuszp_mode: str | None = None


@dataclass
class CompressedBundle:
    segments: tuple[EncodedSegment, ...]
    compressed_size: int
    original_bytes: int


@dataclass
class TransferResult:
    """vLLM's ``TransferResult`` fields (vllm.v1.kv_offload.worker.worker)."""

    job_id: int
    success: bool
    transfer_size: int | None = None
    transfer_time: float | None = None
    transfer_type: Any = None


# --------------------------------------------------------------------------
# On-host job format


class JobHeader:
    """Header and page table at the start of a job's slab.

    Layout (little-endian): magic b"CKVJ", u16 version, u16 element type
    (0 BF16), u32 page count, u64 elements per page, u64 payload bytes, f32
    requested bound, u32 flags (bit 0: relative bound; bits 1-2: codec, 0 cuSZp
    fixed mode, 1 INT8, 2 raw), u32 segments per
    page (G), u32 layer prefix count, u32 source layers (L; 0 when G = 1),
    u64 elements per coded page (G = 1: the page zero-padded to the codec's
    minimum, MIN_CUSZP_ELEMENTS; 0 when G > 1).  When G > 1 a layer table
    follows: L u8 segment indices (the segment that holds each layer, padded
    to 4 bytes) and G f32 requested bounds.  Then per page and segment (entry
    i*G + g) u64 offset (from the payload start), u64 size, f32 absolute
    bound, u32 flags (bit 0: the entry holds the raw BF16 bytes); the payload
    starts at the next 256-byte boundary.  A segment of G > 1 holds the
    page's layers of that segment, in ascending layer order, as
    compress_batch_fixed_bf16_indexed encodes them (or their raw bytes).  An
    INT8 entry is the page's n int8 values and its FP32 scale at byte
    align4(n) (its bound field is 0: the scale is in the payload).
    """

    MAGIC = b"CKVJ"
    VERSION = 3
    RAW = 1
    CODECS = ("cuszp", "int8", "raw")
    _HEAD = struct.Struct("<4sHHIQQfIIIIQ")
    _PAGE = np.dtype([("offset", "<u8"), ("size", "<u8"), ("bound", "<f4"), ("flags", "<u4")])

    @staticmethod
    def _layer_table_bytes(segments: int, layers: int) -> int:
        return 0 if segments <= 1 else (layers + 3) // 4 * 4 + 4 * segments

    @classmethod
    def bytes_for(cls, count: int, segments: int = 1, layers: int = 0) -> int:
        return (cls._HEAD.size + cls._layer_table_bytes(segments, layers) +
                count * segments * cls._PAGE.itemsize + 255) // 256 * 256

    @classmethod
    def write(cls, slab: torch.Tensor, n: int, eps: float, relative: bool, offsets, sizes,
              bounds, payload_bytes: int, groups=None, prefix: int = 0,
              layers: int = 0, raw=None, coded: int = 0, codec: str = "cuszp") -> None:
        """`groups`: None for whole pages, else [(requested bound, layer
        indices)] per segment, the pages viewed as [prefix, layers, n /
        (prefix * layers)].  `raw`: per entry, whether it holds raw bytes.
        `coded`: elements per coded page (whole pages; default n)."""
        segs = 1 if not groups else len(groups)
        count = len(offsets) // segs
        buf = slab[: cls.bytes_for(count, segs, layers)].numpy()
        buf[: cls._HEAD.size] = np.frombuffer(
            cls._HEAD.pack(cls.MAGIC, cls.VERSION, 0, count, n, payload_bytes, eps,
                           (1 if relative else 0) | (cls.CODECS.index(codec) << 1), segs,
                           prefix if segs > 1 else 0,
                           layers if segs > 1 else 0, (coded or n) if segs == 1 else 0),
            dtype=np.uint8)
        start = cls._HEAD.size
        if segs > 1:
            owner = np.zeros((layers + 3) // 4 * 4, dtype=np.uint8)
            for g, (_b, sel) in enumerate(groups):
                owner[list(sel)] = g
            req = np.array([b for b, _sel in groups], dtype="<f4")
            buf[start:start + owner.size] = owner
            buf[start + owner.size:start + owner.size + req.nbytes] = req.view(np.uint8)
            start += owner.size + req.nbytes
        table = np.zeros(count * segs, dtype=cls._PAGE)
        table["offset"] = np.ctypeslib.as_array(offsets)
        table["size"] = np.ctypeslib.as_array(sizes)
        table["bound"] = np.ctypeslib.as_array(bounds)
        if raw is not None:
            table["flags"] = np.asarray(raw, dtype=bool).astype(np.uint32) * cls.RAW
        buf[start:start + table.nbytes] = table.view(np.uint8)

    @classmethod
    def read(cls, slab: torch.Tensor) -> dict:
        """The job's description, validated against the slab."""
        raw = slab[: cls._HEAD.size].numpy().tobytes()
        if len(raw) < cls._HEAD.size:
            raise ValueError("slab shorter than a job header")
        (magic, version, etype, count, n, payload, eps, flags, segs, prefix,
         layers, coded) = cls._HEAD.unpack(raw)
        if magic != cls.MAGIC or version != cls.VERSION or etype != 0:
            raise ValueError("not a compressed KV job (bad magic, version or element type)")
        if segs == 0 or (segs > 1 and (prefix == 0 or layers < segs or
                                       n % (prefix * layers))) or (segs == 1 and coded < n):
            raise ValueError("bad segment description")
        hdr = cls.bytes_for(count, segs, layers)
        if slab.numel() < hdr + payload:
            raise ValueError("slab shorter than its header says")
        start = cls._HEAD.size
        groups = None
        if segs > 1:
            owner = slab[start:start + layers].numpy().copy()
            start += (layers + 3) // 4 * 4
            req = np.frombuffer(slab[start:start + 4 * segs].numpy().tobytes(), dtype="<f4")
            start += 4 * segs
            if np.any(owner >= segs):
                raise ValueError("layer table names a missing segment")
            groups = [(float(req[g]), tuple(int(x) for x in np.flatnonzero(owner == g)))
                      for g in range(segs)]
            if any(not sel for _b, sel in groups):
                raise ValueError("empty segment in the layer table")
        table = np.frombuffer(slab[start:start + count * segs * cls._PAGE.itemsize]
                              .numpy().tobytes(), dtype=cls._PAGE)
        if np.any(table["offset"] + table["size"] > payload) or np.any(table["size"] == 0):
            raise ValueError("page table points outside the payload")
        raw_entries = (table["flags"] & cls.RAW) != 0
        seg_elems = ([n] if segs == 1 else
                     [prefix * len(sel) * (n // (prefix * layers)) for _b, sel in groups])
        want = np.tile(np.asarray(seg_elems, dtype=np.uint64) * 2, count)
        codec_id = (flags >> 1) & 3
        if codec_id >= len(cls.CODECS) or (codec_id and segs != 1):
            raise ValueError("bad codec")
        codec = cls.CODECS[codec_id]
        if codec == "raw":
            raw_entries = np.ones(count, dtype=bool)
        if np.any(raw_entries & (table["size"] != want)):
            raise ValueError("raw entry of the wrong size")
        if codec == "int8" and np.any(table["size"] != (n + 3) // 4 * 4 + 4):
            raise ValueError("INT8 entry of the wrong size")
        return {"count": count, "n": n, "eps": eps, "relative": bool(flags & 1), "codec": codec,
                "segments": segs, "prefix": prefix, "layers": layers, "groups": groups,
                "coded": coded, "payload_at": hdr, "payload_bytes": payload,
                "offsets": table["offset"].astype(np.uint64),
                "sizes": table["size"].astype(np.uint64),
                "bounds": table["bound"].astype(np.float32),
                "raw": raw_entries}


# --------------------------------------------------------------------------
# Host storage (vllm_v1_compressed_offload.py:360-457)


@dataclass
class _Slab:
    buffer: torch.Tensor             # pinned
    payload_at: int = 0              # header and page table bytes
    ticket: int = 0                  # store ticket that fills it
    readers: int = 0                 # last restore ticket reading it
    pages: set[int] = field(default_factory=set)
    # the job's CPU block ids and its page table (offsets, sizes, bounds,
    # raw flags: count x segments), for a load of the same blocks
    job: tuple | None = None


@dataclass
class _PageRecord:
    slab: int
    offsets: tuple[int, ...]         # per segment, from the slab's payload start
    sizes: tuple[int, ...]
    bounds: tuple[float, ...]
    n: int
    raw: tuple[bool, ...] = ()       # per segment: raw BF16 bytes instead of a cuSZp stream


def _ptr_array(addrs: np.ndarray) -> C.Array:
    return (C.c_void_p * len(addrs)).from_buffer_copy(np.asarray(addrs, dtype=np.uint64).tobytes())


class _PageRefs:
    """The destination pages of a restore: their addresses for the pipeline
    (computed in one vector operation, no per-page tensor indexing), and a
    1-D tensor view made only for the entries that need one (raw segments,
    padded pages)."""

    def __init__(self, ptrs: np.ndarray, tensor_of):
        self.ptrs = np.asarray(ptrs, dtype=np.uint64)
        self._tensor_of = tensor_of

    @classmethod
    def of_blocks(cls, kv: torch.Tensor, page_bytes: int, block_ids: np.ndarray) -> "_PageRefs":
        ids = np.asarray(block_ids, dtype=np.int64)
        ptrs = np.uint64(kv.data_ptr()) + ids.astype(np.uint64) * np.uint64(page_bytes)
        return cls(ptrs, lambda i: kv[int(ids[i])].view(-1))

    @classmethod
    def of_tensors(cls, pages: Sequence[torch.Tensor]) -> "_PageRefs":
        flat = [p.view(-1) for p in pages]
        return cls(np.array([p.data_ptr() for p in flat], dtype=np.uint64), lambda i: flat[i])

    def __len__(self) -> int:
        return len(self.ptrs)

    def tensor(self, i: int) -> torch.Tensor:
        return self._tensor_of(int(i))

    def ptr_array(self, sel=None) -> C.Array:
        return _ptr_array(self.ptrs if sel is None else self.ptrs[sel])


def prefault_pinned(buffers: Sequence[torch.Tensor], device, piece: int = 256 << 20) -> None:
    """Runs one DMA pass each way over page-locked host buffers (through a
    device scratch buffer of `piece` bytes), so that a job's first copies
    into or out of a freshly allocated buffer run at the speed of later
    ones: a fresh 1 GiB page-locked buffer was measured to move its first
    pass of copies at about half speed."""
    bufs = [b.view(-1).view(torch.uint8) for b in buffers if b.numel()]
    if not bufs:
        return
    dev = torch.device(device)
    scratch = torch.empty(min(piece, max(b.numel() for b in bufs)), dtype=torch.uint8, device=dev)
    for b in bufs:
        for off in range(0, b.numel(), scratch.numel()):
            n = min(scratch.numel(), b.numel() - off)
            scratch[:n].copy_(b[off:off + n], non_blocking=True)
            b[off:off + n].copy_(scratch[:n], non_blocking=True)
    torch.cuda.synchronize(dev)


class CompressedPageStore:
    """Host storage for compressed pages, shared by both transfer directions.

    ``put_many_packed`` / ``get`` keep the reference's names.  A job's pages
    live in one pinned slab from a pool; a slab goes back to the pool when
    none of its pages is referenced any more (overwritten or evicted)."""

    def __init__(self, allocate=None):
        # page-locked host buffers by default (the pipeline's copies need them)
        self._allocate = allocate or (
            lambda n: torch.empty(n, dtype=torch.uint8, pin_memory=True))
        self._pages: dict[int, _PageRecord] = {}
        self._bundles: dict[int, CompressedBundle] = {}
        self._slabs: dict[int, _Slab] = {}
        self._free: list[tuple[torch.Tensor, int]] = []   # (buffer, last reader ticket)
        self._next_slab = 0
        self._lock = threading.Lock()

    # -- slabs
    def _take_slab(self, nbytes: int, payload_at: int, settle) -> int:
        """A slab of at least nbytes; `settle(ticket)` waits on the host
        for the last restore that read a recycled buffer."""
        with self._lock:
            best = None
            for i, (buf, _t) in enumerate(self._free):
                if buf.numel() >= nbytes and (best is None or
                                               buf.numel() < self._free[best][0].numel()):
                    best = i
            buf, last = self._free.pop(best) if best is not None else (None, 0)
            sid = self._next_slab
            self._next_slab += 1
        if buf is None:
            buf = self._allocate(nbytes)
        elif last:
            settle(last)   # its header is rewritten on the host right away
        with self._lock:
            self._slabs[sid] = _Slab(buf, payload_at)
        return sid

    def reserve(self, nbytes: int, count: int, device=None) -> None:
        """Puts `count` slabs of `nbytes` into the pool ahead of the first
        jobs (a job takes the smallest free slab that holds it), prefaulted
        on `device` when given, so the first jobs neither allocate
        page-locked memory nor run their copies at first-use speed."""
        bufs = [self._allocate(nbytes) for _ in range(count)]
        if device is not None:
            prefault_pinned(bufs, device)
        with self._lock:
            self._free.extend((b, 0) for b in bufs)

    def slab(self, sid: int) -> _Slab:
        return self._slabs[sid]

    def _drop(self, cpu_block_id: int) -> None:
        rec = self._pages.pop(cpu_block_id, None)
        self._bundles.pop(cpu_block_id, None)
        if rec is None:
            return
        slab = self._slabs[rec.slab]
        slab.pages.discard(cpu_block_id)
        if not slab.pages:
            del self._slabs[rec.slab]
            self._free.append((slab.buffer, max(slab.readers, slab.ticket)))

    # -- the reference's interface
    def put_many_packed(self, entries: Iterable[tuple[int, _PageRecord, CompressedBundle]]) -> None:
        with self._lock:
            for cpu_block_id, rec, bundle in entries:
                self._drop(cpu_block_id)
                self._pages[cpu_block_id] = rec
                self._bundles[cpu_block_id] = bundle
                self._slabs[rec.slab].pages.add(cpu_block_id)

    def get(self, cpu_block_id: int) -> CompressedBundle:
        with self._lock:
            bundle = self._bundles.get(cpu_block_id)
        if bundle is None:
            raise KeyError(f"compressed bundle not found for CPU block {cpu_block_id}")
        return bundle

    def record(self, cpu_block_id: int) -> _PageRecord:
        with self._lock:
            rec = self._pages.get(cpu_block_id)
        if rec is None:
            raise KeyError(f"compressed bundle not found for CPU block {cpu_block_id}")
        return rec

    def evict(self, cpu_block_ids: Iterable[int]) -> None:
        with self._lock:
            for b in cpu_block_ids:
                self._drop(int(b))

    def __len__(self) -> int:
        return len(self._pages)


# --------------------------------------------------------------------------
# Handlers (vllm_v1_compressed_offload.py:481-2470)


def _block_ids(spec: Any) -> np.ndarray:
    ids = getattr(spec, "block_ids", spec)
    return np.asarray(ids, dtype=np.int64).reshape(-1)


class _Engine:
    """One libckv context and pipeline per KV cache, shared by both handlers.

    With `layer_bounds` (layer -> requested bound, the reference's
    ``active_bounds`` of ``_compress_adaptive_fixed_bundles_indexed``,
    vllm_v1_compressed_offload.py:1286-1569) a page is viewed as
    ``[layer_prefix, len(layer_bounds), n / (layer_prefix * layers)]`` and
    stored as one segment per distinct bound, in ascending bound order (the
    reference's ``sorted(grouped.items())``); layers missing from the mapping
    take `error_bound`.  One distinct bound leaves whole pages.  Layers of
    bound zero form a segment stored raw (:1381-1409), and a zero bound for
    whole pages stores them raw (:639-656).  Whole pages smaller than
    MIN_CUSZP_ELEMENTS are coded zero-padded to it, as the reference's batched
    path pads them (:904-909).  A KV cache with byte backing storage (uint8 /
    int8) is read as the BF16 pages it holds (:1330-1334)."""

    def __init__(self, kv_cache: torch.Tensor, error_bound: float, device_id: int,
                 chunk_pages: int, layer_bounds=None, layer_prefix: int = 2,
                 codec: str = "cuszp"):
        if kv_cache.dtype in (torch.uint8, torch.int8) and kv_cache.is_contiguous():
            # byte backing storage of BF16 pages (vllm_v1_compressed_offload.py:1330-1334)
            kv_cache = kv_cache.view(torch.uint8).view(kv_cache.shape[0], -1).view(torch.bfloat16)
        if kv_cache.dtype != torch.bfloat16 or not kv_cache.is_cuda or not kv_cache.is_contiguous():
            raise ValueError("kv_cache must be a contiguous BF16 CUDA tensor [num_blocks, ...]")
        if codec not in JobHeader.CODECS:
            raise ValueError(f"unsupported offload codec: {codec}")
        if codec != "cuszp" and layer_bounds is not None:
            raise ValueError("layer bounds apply to the cuSZp codec only")
        self.codec = codec
        self.lib = _ckv.load()
        self.kv = kv_cache
        self.device = kv_cache.device
        self.n = kv_cache[0].numel()
        self.page_bytes = self.n * 2
        self.error_bound = float(error_bound)
        self._set_groups(layer_bounds, int(layer_prefix))
        if self.codec == "cuszp" and self.groups is None and self.error_bound <= 0:
            self.codec = "raw"   # a zero bound stores raw bytes (:639-656)
        self.coded = (max(self.n, MIN_CUSZP_ELEMENTS)
                      if self.groups is None and self.codec == "cuszp" else self.n)
        self.ctx = C.c_void_p()
        # (the context's bound is a default only: every call passes its bounds)
        cfg = _ckv.Config(self.error_bound if self.error_bound > 0 else 1e-4, 1, _ckv.DIM_1D,
                          _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
        self._check(self.lib.ckv_create(cfg, int(device_id), C.byref(self.ctx)), "ckv_create")
        self.pipe = C.c_void_p()
        self._check(self.lib.ckv_pipe_create(self.ctx, int(chunk_pages), C.byref(self.pipe)),
                    "ckv_pipe_create")
        self.lock = threading.Lock()
        self._held: list[tuple[torch.cuda.Event, list[torch.Tensor]]] = []

    def _set_groups(self, layer_bounds, prefix: int) -> None:
        self.groups = None          # [(requested bound, layer indices)] per segment
        self.segments = 1
        self.prefix = self.layers = self.epl = 0
        if layer_bounds is None:
            return
        if isinstance(layer_bounds, dict):
            layers = len(layer_bounds)
            bound_of = [float(layer_bounds.get(i, self.error_bound)) for i in range(layers)]
        else:
            bound_of = [float(b) for b in layer_bounds]
            layers = len(bound_of)
        if layers == 0 or prefix <= 0 or self.n % (prefix * layers):
            raise ValueError("page does not split into [layer_prefix, layers, elements] rows")
        grouped: dict[float, list[int]] = {}
        for layer, bound in enumerate(bound_of):
            grouped.setdefault(max(bound, 0.0), []).append(layer)
        if len(grouped) == 1:
            # one bound: whole pages (a zero bound: raw pages)
            self.error_bound = next(iter(grouped))
            return
        groups = [(b, tuple(sel)) for b, sel in sorted(grouped.items())]
        epl = self.n // (prefix * layers)
        if any(b > 0 and prefix * len(sel) * epl < MIN_CUSZP_ELEMENTS for b, sel in groups):
            raise ValueError(f"a layer segment is smaller than {MIN_CUSZP_ELEMENTS} elements")
        self.groups = groups
        self.segments = len(groups)
        self.prefix, self.layers, self.epl = prefix, layers, epl
        self._index = [torch.tensor(sel, dtype=torch.int64, device=self.device)
                       for _b, sel in self.groups]
        # segments of zero bound are stored raw (:1381-1409); the others through the pipeline
        self.cg = [g for g, (b, _sel) in enumerate(groups) if b > 0]
        Gc = len(self.cg)
        self.sel = (C.c_size_t * Gc)(*[len(groups[g][1]) for g in self.cg])
        self.idx = (C.c_void_p * Gc)(*[self._index[g].data_ptr() for g in self.cg])
        self.eps = (C.c_float * Gc)(*[groups[g][0] for g in self.cg])

    def segment_numel(self, g: int) -> int:
        return self.n if self.groups is None else self.prefix * len(self.groups[g][1]) * self.epl

    def segment_bytes(self, page: torch.Tensor, g: int) -> torch.Tensor:
        """The raw bytes of segment g of a page (a device tensor)."""
        if self.groups is None:
            return page.reshape(-1).view(torch.uint8)
        view = page.reshape(self.prefix, self.layers, self.epl)
        return view.index_select(1, self._index[g]).contiguous().view(-1).view(torch.uint8)

    def _check(self, status: int, what: str) -> None:
        if status != 0:
            raise RuntimeError(f"{what}: {_ckv.error_message(self.lib, self.ctx, status)}")

    def page_ptrs(self, block_ids: np.ndarray) -> C.Array:
        if block_ids.size and (block_ids.min() < 0 or block_ids.max() >= self.kv.shape[0]):
            raise IndexError("GPU block id out of range")
        addrs = np.uint64(self.kv.data_ptr()) + block_ids.astype(np.uint64) * np.uint64(self.page_bytes)
        return (C.c_void_p * len(addrs)).from_buffer_copy(addrs.astype(np.uint64).tobytes())

    def host_capacity(self, count: int) -> int:
        if self.codec == "int8":
            return int(self.lib.ckv_pipe_host_capacity_int8(count, self.n))
        if self.codec == "raw":
            return int(self.lib.ckv_pipe_host_capacity_raw(count, self.page_bytes))
        if self.groups is None:
            return int(self.lib.ckv_pipe_host_capacity(count, self.coded))
        raw = sum((2 * self.segment_numel(g) + 15) // 16 * 16
                  for g in range(self.segments) if g not in self.cg)
        return int(self.lib.ckv_pipe_host_capacity_groups(count, self.sel, len(self.cg),
                                                          self.prefix, self.epl)) + count * raw

    def store(self, pages: C.Array, count: int, eps: float, host: int, cap: int, offsets,
              sizes, bounds, total, after: int, ticket, stream: int) -> None:
        if self.codec == "int8":
            self._check(self.lib.ckv_pipe_store_int8(
                self.pipe, pages, count, self.n, host, cap, offsets, sizes, total, after, ticket,
                stream), "store")
        elif self.codec == "raw":
            self._check(self.lib.ckv_pipe_store_raw(
                self.pipe, pages, count, self.page_bytes, host, cap, offsets, total, after, ticket,
                stream), "store")
            for i in range(count):
                sizes[i] = self.page_bytes
        elif self.groups is None:
            self._check(self.lib.ckv_pipe_store_bf16(
                self.pipe, pages, (C.c_float * count)(*([eps] * count)), count, self.coded, host,
                cap, offsets, sizes, bounds, total, after, ticket, stream), "store")
        else:
            # the compressed segments (entry i * Gc + j); the caller places raw ones
            self._check(self.lib.ckv_pipe_store_bf16_groups(
                self.pipe, pages, count, self.idx, self.sel, len(self.cg), self.prefix,
                self.layers, self.epl, self.eps, host, cap, offsets, sizes, bounds, total,
                after, ticket, stream), "store")

    def join(self, ticket: int, stream: int) -> None:
        self._check(self.lib.ckv_pipe_join(self.pipe, ticket, stream), "join")

    def record(self, stream: int) -> int:
        t = C.c_uint64(0)
        self._check(self.lib.ckv_pipe_record(self.pipe, stream, C.byref(t)), "record")
        return t.value

    def hold(self, tensors: list[torch.Tensor], stream) -> None:
        """Keeps device tensors the pipeline's own streams use alive until the
        work queued on `stream` (ordered after them) is done."""
        self._held = [(ev, ts) for ev, ts in self._held if not ev.query()]
        if tensors:
            ev = torch.cuda.Event()
            ev.record(stream)
            self._held.append((ev, tensors))

    def restore(self, payload: torch.Tensor, offsets, sizes, bounds, raw, dst: _PageRefs,
                after: int, stream) -> int:
        """Restores a job's entries (page i, segment g at i * G + g) from
        `payload` (the pinned bytes after the job header) into the pages
        `dst`: cuSZp entries through the pipeline, raw entries by copies,
        padded pages through a staging buffer.  Returns a ticket that covers
        all of it."""
        G, count = self.segments, len(dst)
        sptr = stream.cuda_stream
        if self.codec != "cuszp":
            t = C.c_uint64(0)
            offs = (C.c_size_t * count)(*[int(o) for o in offsets])
            ptrs = dst.ptr_array()
            if self.codec == "int8":
                self._check(self.lib.ckv_pipe_restore_int8(
                    self.pipe, payload.data_ptr(), offs, count, self.n, ptrs, after, C.byref(t),
                    sptr), "restore")
            else:
                self._check(self.lib.ckv_pipe_restore_raw(
                    self.pipe, payload.data_ptr(), offs, count, self.page_bytes, ptrs, after,
                    C.byref(t), sptr), "restore")
            return t.value
        offsets = np.asarray(offsets, dtype=np.uint64).reshape(count, G)
        sizes = np.asarray(sizes, dtype=np.uint64).reshape(count, G)
        bounds = np.asarray(bounds, dtype=np.float32).reshape(count, G)
        raw = np.asarray(raw, dtype=bool).reshape(count, G)
        base = payload.data_ptr()
        tickets, held, extra = [], [], False

        def arrays(sel, g=None):
            cols = slice(None) if g is None else slice(g, g + 1)
            o, z, b = offsets[sel][:, cols], sizes[sel][:, cols], bounds[sel][:, cols]
            k = o.size
            return ((C.c_size_t * k)(*o.reshape(-1).tolist()), (C.c_size_t * k)(*z.reshape(-1).tolist()),
                    (C.c_float * k)(*b.reshape(-1).tolist()))

        cg = [0] if G == 1 else self.cg
        comp = ~raw[:, cg]
        if G == 1 or comp.all():
            sel = np.flatnonzero(comp.all(axis=1))
            if sel.size:
                t = C.c_uint64(0)
                if G == 1:
                    o, z, b = arrays(sel)
                    if self.coded > self.n:
                        stage = torch.empty(len(sel), self.coded, dtype=torch.bfloat16,
                                            device=self.device)
                        held.append(stage)
                        ptrs = _ckv.ptr_array([stage[k].data_ptr() for k in range(len(sel))])
                    else:
                        ptrs = dst.ptr_array(sel)
                    self._check(self.lib.ckv_pipe_restore_bf16(
                        self.pipe, base, o, z, b, len(sel), self.coded, ptrs, after,
                        C.byref(t), sptr), "restore")
                    if self.coded > self.n:
                        self.join(t.value, sptr)
                        for k, i in enumerate(sel):
                            dst.tensor(i).copy_(stage[k, :self.n])
                        extra = True
                else:
                    k = len(sel) * len(cg)
                    o = (C.c_size_t * k)(*offsets[sel][:, cg].reshape(-1).tolist())
                    z = (C.c_size_t * k)(*sizes[sel][:, cg].reshape(-1).tolist())
                    b = (C.c_float * k)(*bounds[sel][:, cg].reshape(-1).tolist())
                    self._check(self.lib.ckv_pipe_restore_bf16_groups(
                        self.pipe, base, o, z, b, len(sel), self.idx, self.sel, len(cg),
                        self.prefix, self.layers, self.epl, dst.ptr_array(sel), after,
                        C.byref(t), sptr), "restore")
                tickets.append(t.value)
        else:
            # some compressed segments were stored raw: each group's cuSZp
            # segments in a call of their own
            for j, g in enumerate(cg):
                sel = np.flatnonzero(comp[:, j])
                if not sel.size:
                    continue
                o, z, b = arrays(sel, g)
                t = C.c_uint64(0)
                self._check(self.lib.ckv_pipe_restore_bf16_groups(
                    self.pipe, base, o, z, b, len(sel), (C.c_void_p * 1)(self.idx[j]),
                    (C.c_size_t * 1)(self.sel[j]), 1, self.prefix, self.layers, self.epl,
                    dst.ptr_array(sel), after, C.byref(t), sptr),
                    "restore")
                tickets.append(t.value)
        if raw.any():
            # raw entries: copied from the page-locked payload after the store that wrote it
            self.join(after, sptr)
            with torch.cuda.stream(stream):
                for i, g in zip(*np.nonzero(raw)):
                    o, nbytes = int(offsets[i, g]), 2 * self.segment_numel(g)
                    src = payload[o:o + nbytes]
                    if self.groups is None:
                        dst.tensor(i).view(torch.uint8).copy_(src, non_blocking=True)
                    else:
                        tmp = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                        tmp.copy_(src, non_blocking=True)
                        dst.tensor(i).view(self.prefix, self.layers, self.epl).index_copy_(
                            1, self._index[g],
                            tmp.view(torch.bfloat16).view(self.prefix, len(self.groups[g][1]),
                                                          self.epl))
            extra = True
        if len(tickets) == 1 and not extra:
            final = tickets[0]
        else:
            for t in tickets:
                self.join(t, sptr)
            final = self.record(sptr)
        self.hold(held, stream)
        return final

    def close(self) -> None:
        if self.pipe:
            self.lib.ckv_pipe_destroy(self.pipe)
            self.pipe = C.c_void_p()
        if self.ctx:
            self.lib.ckv_destroy(self.ctx)
            self.ctx = C.c_void_p()
        self._held = []


class CompressedOffloadingHandler:
    """One transfer direction.  ``transfer_async(job_id, (src_spec, dst_spec))``
    with GPU block ids on the GPU side and CPU block ids (keys of the page
    store) on the CPU side.

    Each direction issues its jobs on a CUDA stream of its own, ordered after
    the work already on the caller's current stream (the model's writes to
    the blocks), and never makes the caller's stream wait: as in the
    reference (vllm_v1_compressed_offload.py:2365-2385, a worker thread's
    stream after a ready event), a job's blocks are the caller's again once
    get_finished reports it or wait returns.  So a store and a load issued
    one after the other overlap instead of queueing behind each other, and
    jobs of one direction run in issue order."""

    def __init__(self, engine: _Engine, store: CompressedPageStore, gpu_to_cpu: bool,
                 error_bound: float | None = None):
        self.engine = engine
        self.store = store
        self.gpu_to_cpu = bool(gpu_to_cpu)
        self.error_bound = float(engine.error_bound if error_bound is None else error_bound)
        self.transfer_type = ("GPU", "CPU") if gpu_to_cpu else ("CPU", "GPU")
        self._pending: dict[int, tuple[list[int], int]] = {}   # job -> (tickets, bytes)
        self._finished: list[TransferResult] = []
        self._lock = threading.Lock()
        self._finalize: dict[int, list] = {}   # INT8 store ticket -> its page entries
        self._stream: torch.cuda.Stream | None = None           # created by the first job

    def _components(self, g: int) -> tuple[BundleComponent, ...]:
        e = self.engine
        if e.groups is None:
            return (BundleComponent(0, tuple(e.kv.shape[1:]), torch.bfloat16, e.n),)
        sel = e.groups[g][1]
        return (BundleComponent(0, (e.prefix, len(sel), e.epl), torch.bfloat16,
                                e.segment_numel(g), layer_axis=1, layer_indices=sel,
                                destination_view_shape=(e.prefix, e.layers, e.epl)),)

    # -- one job
    def _store(self, gpu_ids: np.ndarray, cpu_ids: np.ndarray) -> tuple[list[int], int]:
        e = self.engine
        count, G = len(gpu_ids), e.segments
        stream = torch.cuda.current_stream(e.device)
        if e.coded > e.n:
            # small pages, zero-padded to the codec's minimum (vllm_v1_compressed_offload.py:904-909)
            src = torch.zeros(count, e.coded, dtype=torch.bfloat16, device=e.device)
            src[:, :e.n] = e.kv.view(e.kv.shape[0], -1)[torch.as_tensor(gpu_ids, device=e.device)]
            pages = _ckv.ptr_array([src[i].data_ptr() for i in range(count)])
        else:
            pages = e.page_ptrs(gpu_ids)
        hdr = JobHeader.bytes_for(count, G, e.layers)
        cap = e.host_capacity(count)
        sid = self.store._take_slab(hdr + cap, hdr,
                                    lambda t: e._check(e.lib.ckv_pipe_wait(e.pipe, t), "wait"))
        slab = self.store.slab(sid)
        offsets = (C.c_size_t * (count * G))()
        sizes = (C.c_size_t * (count * G))()
        bounds = (C.c_float * (count * G))()
        total = C.c_size_t(0)
        ticket = C.c_uint64(0)
        cg = [0] if e.groups is None else e.cg
        if len(cg) == G:
            e.store(pages, count, self.error_bound, slab.buffer.data_ptr() + hdr, cap, offsets,
                    sizes, bounds, C.byref(total), slab.readers, C.byref(ticket), stream.cuda_stream)
        else:
            Gc = len(cg)
            co, cs = (C.c_size_t * (count * Gc))(), (C.c_size_t * (count * Gc))()
            cb = (C.c_float * (count * Gc))()
            e.store(pages, count, self.error_bound, slab.buffer.data_ptr() + hdr, cap, co, cs, cb,
                    C.byref(total), slab.readers, C.byref(ticket), stream.cuda_stream)
            pos = (total.value + 15) // 16 * 16
            for i in range(count):
                for j, g in enumerate(cg):
                    offsets[i * G + g] = co[i * Gc + j]
                    sizes[i * G + g] = cs[i * Gc + j]
                    bounds[i * G + g] = cb[i * Gc + j]
                for g in (g for g in range(G) if g not in cg):
                    offsets[i * G + g] = pos
                    sizes[i * G + g] = 2 * e.segment_numel(g)
                    pos += (sizes[i * G + g] + 15) // 16 * 16
            total.value = pos
        final = ticket.value
        # A page (segment) that cuSZp would not shrink below its raw BF16 size is
        # stored raw, with bound 0 (vllm_v1_compressed_offload.py:1000-1010): its
        # raw bytes fit where its longer stream was packed.
        seg_bytes = [2 * e.segment_numel(g) for g in range(G)]
        raw = [e.codec == "raw" or (e.codec == "cuszp" and (j % G not in cg or
                                                             int(sizes[j]) >= seg_bytes[j % G]))
               for j in range(count * G)]
        if e.codec == "cuszp" and any(raw):
            e.join(final, stream.cuda_stream)
            with torch.cuda.stream(stream):
                for j in (j for j in range(count * G) if raw[j]):
                    i, g = divmod(j, G)
                    src_bytes = e.segment_bytes(e.kv[int(gpu_ids[i])], g)
                    at = hdr + int(offsets[j])
                    slab.buffer[at:at + seg_bytes[g]].copy_(src_bytes, non_blocking=True)
                    sizes[j] = seg_bytes[g]
                    bounds[j] = 0.0
            final = e.record(stream.cuda_stream)
        slab.ticket = final
        slab.job = (np.asarray(cpu_ids, dtype=np.int64).copy(),
                    np.ctypeslib.as_array(offsets).reshape(count, G).copy(),
                    np.ctypeslib.as_array(sizes).reshape(count, G).copy(),
                    np.ctypeslib.as_array(bounds).reshape(count, G).copy(),
                    np.asarray(raw, dtype=bool).reshape(count, G))
        JobHeader.write(slab.buffer, e.n, self.error_bound, True, offsets, sizes, bounds,
                        total.value, e.groups, e.prefix, e.layers, raw=raw, coded=e.coded,
                        codec=e.codec)
        comps = [self._components(g) for g in range(G)]
        req = [self.error_bound] if e.groups is None else [b for b, _sel in e.groups]
        numels = [e.segment_numel(g) for g in range(G)]
        codeds = [e.coded if e.groups is None else numels[g] for g in range(G)]
        # the page table as Python lists once: per-page records are then
        # plain slices (the job's host bookkeeping runs while its copies fly)
        ids_l, offs_l, sizes_l = slab.job[0].tolist(), slab.job[1].ravel().tolist(), \
            slab.job[2].ravel().tolist()
        bounds_l, buf = slab.job[3].ravel().tolist(), slab.buffer
        entries = []
        for i in range(count):
            j0, j1 = i * G, i * G + G
            ro, rs, rr = tuple(offs_l[j0:j1]), tuple(sizes_l[j0:j1]), tuple(raw[j0:j1])
            rb = tuple(bounds_l[j0:j1])
            rec = _PageRecord(sid, ro, rs, rb, e.n, rr)
            segs = []
            for g in range(G):
                encoding = "raw" if rr[g] else e.codec
                segs.append(EncodedSegment(buf[hdr + ro[g]: hdr + ro[g] + rs[g]], rs[g], rb[g],
                                           encoding, comps[g], numels[g], codeds[g],
                                           numels[g] * 2, req[g],
                                           cuszp_mode="fixed" if encoding == "cuszp" else None))
            entries.append((ids_l[i], rec,
                            CompressedBundle(tuple(segs), sum(rs), e.page_bytes)))
        self.store.put_many_packed(entries)
        if e.codec == "int8":
            self._finalize[final] = entries
        return [final], int(total.value)

    def _load(self, cpu_ids: np.ndarray, gpu_ids: np.ndarray) -> tuple[list[int], int]:
        e = self.engine
        if gpu_ids.size and (gpu_ids.min() < 0 or gpu_ids.max() >= e.kv.shape[0]):
            raise IndexError("GPU block id out of range")
        stream = torch.cuda.current_stream(e.device)
        # A load of exactly the blocks one store job wrote, all still in its
        # slab, uses that job's page table as stored (no per-page lookups).
        if cpu_ids.size:
            slab = self.store.slab(self.store.record(int(cpu_ids[0])).slab)
            job = slab.job
            if (job is not None and job[1].shape[1] == e.segments and
                    len(job[0]) == len(cpu_ids) and len(slab.pages) == len(cpu_ids) and
                    np.array_equal(job[0], cpu_ids)):
                _ids, offs, sizes, bounds, raw = job
                dst = _PageRefs.of_blocks(e.kv, e.page_bytes, gpu_ids)
                t = e.restore(slab.buffer[slab.payload_at:], offs.reshape(-1), sizes.reshape(-1),
                              bounds.reshape(-1), raw.reshape(-1), dst, slab.ticket, stream)
                slab.readers = t
                return [t], int(sizes.sum())
        recs = [self.store.record(int(c)) for c in cpu_ids]
        if any(len(r.sizes) != e.segments or r.n != e.n for r in recs):
            raise ValueError("stored page does not match the KV cache layout")
        by_slab: dict[int, list[int]] = {}
        for i, r in enumerate(recs):
            by_slab.setdefault(r.slab, []).append(i)
        tickets, nbytes = [], 0
        for sid, idx in by_slab.items():
            slab = self.store.slab(sid)
            offs = [o for i in idx for o in recs[i].offsets]
            sizes = [z for i in idx for z in recs[i].sizes]
            bounds = [b for i in idx for b in recs[i].bounds]
            raw = [r for i in idx for r in (recs[i].raw or (False,) * e.segments)]
            dst = _PageRefs.of_blocks(e.kv, e.page_bytes, gpu_ids[idx])
            t = e.restore(slab.buffer[slab.payload_at:], offs, sizes, bounds, raw, dst,
                          slab.ticket, stream)
            slab.readers = t
            tickets.append(t)
            nbytes += sum(sizes)
        return tickets, nbytes

    # -- the OffloadingHandler interface (vLLM)
    def transfer_async(self, job_id: int, spec: Sequence[Any]) -> bool:
        src, dst = spec
        src_ids, dst_ids = _block_ids(src), _block_ids(dst)
        if len(src_ids) != len(dst_ids):
            raise ValueError("GPU/CPU block specification length mismatch")
        with self.engine.lock:
            if len(src_ids) == 0:
                tickets, nbytes = [], 0
            else:
                dev = self.engine.device
                if self._stream is None:
                    self._stream = torch.cuda.Stream(dev)
                self._stream.wait_stream(torch.cuda.current_stream(dev))
                # _store / _load issue on the current stream, here this direction's
                with torch.cuda.stream(self._stream):
                    if self.gpu_to_cpu:
                        tickets, nbytes = self._store(src_ids, dst_ids)
                    else:
                        tickets, nbytes = self._load(src_ids, dst_ids)
        with self._lock:
            self._pending[int(job_id)] = (tickets, nbytes)
        return True

    def get_finished(self) -> list[TransferResult]:
        """Jobs finished since the last call."""
        lib, pipe = self.engine.lib, self.engine.pipe
        with self._lock:
            done = []
            for job_id, (tickets, nbytes) in self._pending.items():
                states = [lib.ckv_pipe_done(pipe, t) for t in tickets]
                if all(s != 0 for s in states):
                    done.append((job_id, all(s == 1 for s in states), nbytes))
            for job_id, ok, nbytes in done:
                for t in self._pending[job_id][0]:
                    self._scales(t)
                del self._pending[job_id]
                self._finished.append(TransferResult(job_id, ok, nbytes,
                                                     transfer_type=self.transfer_type))
            out, self._finished = self._finished, []
        return out

    def wait(self, job_ids: set[int]) -> None:
        lib, pipe = self.engine.lib, self.engine.pipe
        with self._lock:
            tickets = [t for j in job_ids for t in self._pending.get(int(j), ([], 0))[0]]
        for t in tickets:
            self.engine._check(lib.ckv_pipe_wait(pipe, t), "wait")
            with self._lock:
                self._scales(t)

    def _scales(self, ticket: int) -> None:
        """Once an INT8 store has landed: each page's FP32 scale (at byte
        align4(n) of its stored form) into its metadata, and the bound the
        reference records for it, scale / 2 (vllm_v1_compressed_offload.py:
        711-724)."""
        entries = self._finalize.pop(ticket, None)
        if not entries:
            return
        at = (self.engine.n + 3) // 4 * 4
        for _cpu, rec, bundle in entries:
            seg = bundle.segments[0]
            scale = float(np.frombuffer(seg.payload[at:at + 4].numpy().tobytes(), dtype="<f4")[0])
            seg.quant_scale = scale
            seg.actual_error_bound = scale / 2.0
            rec.bounds = (scale / 2.0,)

    def shutdown(self) -> None:
        with self._lock:
            pending = list(self._pending)
        self.wait(set(pending))


class CompressedCpuGpuOffloadingHandlers:
    """Both directions over one KV cache (vllm_v1_compressed_offload.py:2412-2470).

    `layer_bounds` / `layer_prefix`: a fixed per-layer bound assignment (the
    reference's calibrated mixed profiles, e.g. 1e-5 on a few sensitive
    layers and 1e-4 on the rest), stored as one segment per distinct bound
    (see ``_Engine``).  `codec`: "cuszp" (fixed mode), or the reference
    connector's GPU comparison codecs "int8" (per-page absmax / 127) and
    "raw" (vllm_v1_compressed_offload.py:508-511)."""

    def __init__(self, kv_cache: torch.Tensor, error_bound: float = 1e-4, device_id: int = 0,
                 chunk_pages: int = 64, layer_bounds=None, layer_prefix: int = 2,
                 codec: str = "cuszp"):
        self.engine = _Engine(kv_cache, error_bound, device_id, chunk_pages, layer_bounds,
                              layer_prefix, codec)
        self.store = CompressedPageStore()
        self.gpu_to_cpu_handler = CompressedOffloadingHandler(self.engine, self.store, True)
        self.cpu_to_gpu_handler = CompressedOffloadingHandler(self.engine, self.store, False)

    def shutdown(self) -> None:
        self.gpu_to_cpu_handler.shutdown()
        self.cpu_to_gpu_handler.shutdown()
        self.engine.close()


def restore_job(slab: torch.Tensor, dst_pages: Sequence[torch.Tensor], engine: _Engine) -> int:
    """Restores every page of a job from its slab bytes alone (the header and
    page table), e.g. after the slab was written to a file and read back.
    The job's segments must be the engine's.  Returns the pipeline ticket."""
    job = JobHeader.read(slab)
    if job["n"] != engine.n or len(dst_pages) != job["count"]:
        raise ValueError("job does not match the destination pages")
    if job["codec"] != engine.codec:
        raise ValueError(f"job stored with the {job['codec']} codec, engine uses {engine.codec}")
    same = job["segments"] == engine.segments and (
        (engine.groups is None and job["coded"] == engine.coded) or
        (engine.groups is not None and
         [sel for _b, sel in job["groups"]] == [sel for _b, sel in engine.groups] and
         job["prefix"] == engine.prefix and job["layers"] == engine.layers))
    if not same:
        raise ValueError("job segments do not match the engine's layer groups")
    return engine.restore(slab[job["payload_at"]:], job["offsets"], job["sizes"], job["bounds"],
                          job["raw"], _PageRefs.of_tensors(dst_pages), 0,
                          torch.cuda.current_stream(engine.device))
