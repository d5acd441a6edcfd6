#!/usr/bin/env python
"""Benchmark of the fixed-mode KV-page codec on B200 (one JSON line).

Workload ("C2"): Qwen2.5-1.5B-shaped KV cache at
4k context -- 256 pages of [2 (K/V), 28 layers, 2 KV heads, 16 tokens,
128 head_dim] BF16 = 229376 elements (458752 B) per page, 117.44 MB in all;
REL error bound 1e-5.  Synthetic, seeded on the CPU: K = N(0,1) times a
LogNormal(0, 0.5) scale per (layer, head, channel) with 4 outlier channels
x8, V = N(0, 0.5^2).

One step = store (compress every page, sizes back on the host) + restore
(decompress every page into its KV page).
  value  -- uncompressed bytes through the codec (stored + restored) per
            second, inputs resident in HBM, C-ABI calls (include/ckv.h)
            timed with CUDA events; L2 flushed (256 MB write) between steps.
  e2e    -- the same with host buffers, through the store / restore
            pipeline (ckv_pipe_*): step k's pages are stored into one
            page-locked slab while step k-1's slab is restored.
  roofline -- the dominant kernel's algorithmic bytes (encode 2N + S_c,
            decode S_c + 2N per page) / its CUDA-event duration, against the
            measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline -- the CPU port of the codec (oracle/fixed_codec.c) on all
            host cores, same pages, encode + decode.

--impl reference is the reference arm on the host cores: the reference's
codec is CUDA with no CPU implementation, so the C restatement of its
kernels (oracle/fixed_codec.c) encodes and decodes the same pages on every
host thread (rank 0 alone under torchrun).  The reference's own kernels
(integration/cuszp_wrapper/cuszp_batched_fixed.cu, built unchanged into
oracle/_ref) run on the GPU inside this arm, driven like its CuSZpWrapper
and its connector's packed store / batched restore: `reference_kernels`.

Multi-GPU (torchrun, N ranks): each rank encodes and decodes its own 256
pages (its tensor-parallel KV shard); no data-path collective; value is the
total over ranks divided by the slowest rank's time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import gc
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "reducing-pcie-bottlenecks-for-llm-serving-with-cuszp-compressed-kv-cache-transfer_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT))

METRIC = "effective KV store/restore GB/s per GPU (uncompressed) + ratio; kernel HBM % peak"
LAYERS, HEADS, TOKENS, HEAD_DIM = 28, 2, 16, 128
PAGE_NUMEL = 2 * LAYERS * HEADS * TOKENS * HEAD_DIM  # 229376
PAGES = 256
EPS = 1e-5
FALLBACK_HBM_GBS = 6650.0


def make_pages(pages: int, seed: int) -> torch.Tensor:
    """Seeded synthetic KV pages on the CPU, [pages, PAGE_NUMEL] BF16."""
    g = torch.Generator().manual_seed(seed)
    kscale = torch.empty(LAYERS, HEADS, HEAD_DIM).log_normal_(0.0, 0.5, generator=g)
    outliers = torch.randperm(HEAD_DIM, generator=g)[:4]
    kscale[:, :, outliers] *= 8.0
    out = torch.empty(pages, PAGE_NUMEL, dtype=torch.bfloat16)
    chunk = 32
    for p0 in range(0, pages, chunk):
        p1 = min(pages, p0 + chunk)
        k = torch.randn(p1 - p0, LAYERS, HEADS, TOKENS, HEAD_DIM, generator=g)
        k *= kscale[None, :, :, None, :]
        v = torch.randn(p1 - p0, LAYERS, HEADS, TOKENS, HEAD_DIM, generator=g) * 0.5
        out[p0:p1] = torch.stack([k, v], dim=1).reshape(p1 - p0, -1).to(torch.bfloat16)
    return out


def measured_hbm_gbs() -> tuple[float, str]:
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel: str) -> tuple[float | None, str | None]:
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = ROOT / "profiles" / f"{kernel}_c2.md"
    if not path.exists():
        return None, None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip()), str(path.relative_to(ROOT))
    return None, None


class ClockSampler:
    """SM clock and clock-event reasons sampled every ~2 ms during the timed
    region (the timed regions last milliseconds, far below nvidia-smi's
    polling period), read through NVML; nvidia-smi at 200 ms otherwise."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4}
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device, physical_index: int, period_s: float = 0.002,
                 enabled: bool = True):
        self.enabled = enabled
        self.period = period_s
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.source = None
        self.nvml = None
        self.handle = None
        self.proc = None
        self.lines: list[str] = []
        if not enabled:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(device).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(physical_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                  pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
            self.source = "nvml, 2 ms"
        except Exception:
            self.nvml = None
            self.physical = physical_index

    def _reasons(self) -> int:
        try:
            return int(self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
        except Exception:
            return int(self.nvml.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle))

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = int(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                self.samples.append((float(mhz), self._reasons()))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if not self.enabled:
            return self
        if self.nvml is not None:
            import threading
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.physical)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi, 200 ms"
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if not self.enabled:
            return
        if self.nvml is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            return
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in out.splitlines():
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz, self.max_mhz = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            bits = 0
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    bits |= self.REASONS[name]
            self.samples.append((mhz, bits))

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": self.source}
        reasons = sorted(name for name, bit in self.REASONS.items()
                         if any(b & bit for _, b in self.samples))
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": self.source}


# ---------------------------------------------------------------------------
# CPU baseline: the C port of the codec on all host cores.


def cpu_baseline(host_pages: torch.Tensor, budget_s: float = 10.0) -> dict:
    """The CPU port of the codec (oracle/fixed_codec.c) on all host cores:
    encode + decode of the full C2 batch, repeated for about `budget_s`
    seconds (at least once); the mean over the repetitions."""
    from oracle.oracle import COracle
    co = COracle()
    threads = len(os.sched_getaffinity(0)) or 1
    bits = host_pages.view(torch.int16).numpy().view(np.uint16)
    pages = [np.ascontiguousarray(bits[i]) for i in range(bits.shape[0])]
    n = pages[0].size
    dest = [np.empty(n, dtype=np.uint16) for _ in pages]
    dp = (C.c_void_p * len(dest))(*[d.ctypes.data for d in dest])
    enc_t, dec_t = [], []
    while not enc_t or sum(enc_t) + sum(dec_t) < budget_s:
        t0 = time.perf_counter()
        outs, sizes, ebs = co.encode_batch_bf16(pages, EPS, relative=True, threads=threads)
        enc_t.append(time.perf_counter() - t0)
        ins = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        sz = np.ascontiguousarray(sizes, dtype=np.uint64)
        eb = np.ascontiguousarray(ebs, dtype=np.float32)
        t0 = time.perf_counter()
        rc = co.lib.ckvo_decode_batch_bf16(ins, sz.ctypes.data, eb.ctypes.data, dp,
                                           len(outs), n, threads)
        dec_t.append(time.perf_counter() - t0)
        assert rc == 0
    raw = bits.nbytes
    reps = len(enc_t)
    t = sum(enc_t) + sum(dec_t)
    return {"value": round(2 * raw * reps / t / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{len(pages)} pages x {n} BF16 (the full step), encode + decode, "
                      f"{reps} repetitions ({t:.1f} s), mean; oracle/fixed_codec.c, "
                      f"{threads} threads",
            "store_gbps": round(raw * reps / sum(enc_t) / 1e9, 3),
            "restore_gbps": round(raw * reps / sum(dec_t) / 1e9, 3)}


DIRECTION_KEYS = ("store_gbps", "restore_gbps", "overlapped_gbps", "raw_d2h_gbps",
                  "raw_h2d_gbps", "store_vs_raw_d2h", "restore_vs_raw_h2d", "compression_ratio",
                  "restore_ok")


def per_config_summary(world, line, c2_dirs, e2e, c1_pipe, c3, streamed) -> dict:
    """Every BASELINE.json config with host copies, per direction: the store
    alone and the restore alone (uncompressed GB/s, all ranks) next to raw
    one-way page-locked copies of the same pages, and both directions in
    flight together."""
    out = {}
    if c1_pipe:
        for key in ("jobs_per_call_1", "jobs_per_call_16"):
            if key in c1_pipe:
                out[f"C1_{key}"] = {k: c1_pipe[key].get(k) for k in DIRECTION_KEYS}
    if c2_dirs:
        c2 = {k: c2_dirs.get(k) for k in DIRECTION_KEYS}
        c2["overlapped_gbps"] = round(e2e, 3)
        c2["compression_ratio"] = line.get("compression_ratio")
        c2["restore_ok"] = bool(line.get("store_restore_ok")) and bool(
            line["e2e"].get("restore_matches_kernel_path"))
        out["C2"] = c2
    if c3:
        out["C3"] = {k: c3.get(k) for k in DIRECTION_KEYS}
    for name, leg in (streamed or {}).items():
        out[name] = ({k: leg.get(k) for k in DIRECTION_KEYS} if "skipped" not in leg
                     else {"skipped": leg["skipped"]})
        if "skipped" not in leg:
            out[name]["n_gpus"] = leg.get("n_gpus")
    for name, v in out.items():
        if v.get("restore_gbps") and v.get("raw_h2d_gbps"):
            v["restore_beats_raw_h2d"] = v["restore_gbps"] > v["raw_h2d_gbps"]
    out["n_gpus"] = world
    return out


def config_block(pages: int) -> dict:
    """The workload description both arms print (identical, so the two lines
    compare as the same configuration)."""
    return {"workload": "C2: Qwen2.5-1.5B KV at 4k context, 256 pages x 229376 BF16 "
                        "([2,28,2,16,128]), REL eb 1e-5, one store + one restore per step",
            "pages_per_gpu": pages, "elements_per_page": PAGE_NUMEL,
            "error_bound": EPS, "relative": True,
            "l2_flush": "256 MB write between timed steps",
            "parallelism": "one process per GPU, pages sharded, no data-path collective"}


def reference_arm(args, world: int) -> dict:
    """The reference arm: the reference's path has no CPU implementation of
    its own (its codec is CUDA), so the C restatement of its kernels
    (oracle/fixed_codec.c, checked byte for byte against the reference's
    kernels on the committed goldens) runs on all host cores: W untimed and K
    timed steps, each an encode and a decode of the full C2 batch."""
    from oracle.oracle import COracle
    co = COracle()
    threads = len(os.sched_getaffinity(0)) or 1
    host = make_pages(args.pages, seed=0)
    bits = host.view(torch.int16).numpy().view(np.uint16)
    pages = [np.ascontiguousarray(bits[i]) for i in range(bits.shape[0])]
    n = pages[0].size
    raw = bits.nbytes
    dest = [np.empty(n, dtype=np.uint16) for _ in pages]
    dp = (C.c_void_p * len(dest))(*[d.ctypes.data for d in dest])

    def step():
        outs, sizes, ebs = co.encode_batch_bf16(pages, EPS, relative=True, threads=threads)
        ins = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        sz = np.ascontiguousarray(sizes, dtype=np.uint64)
        eb = np.ascontiguousarray(ebs, dtype=np.float32)
        assert co.lib.ckvo_decode_batch_bf16(ins, sz.ctypes.data, eb.ctypes.data, dp, len(outs),
                                             n, threads) == 0
        return int(sz.sum())

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    comp = 0
    for _ in range(args.steps):
        comp = step()
    t = time.perf_counter() - t0
    value = round(2 * raw * args.steps / t / 1e9, 3)
    sample = (f"{len(pages)} pages x {n} BF16 per step (the full C2 batch), encode + decode; "
              f"oracle/fixed_codec.c on {threads} host threads")
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32/u32",
        "data": "synthetic (seeded CPU generation, BASELINE.json configs[1] shapes)",
        "config": config_block(args.pages),
        "compression_ratio": round(raw / max(1, comp), 4),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "host": host_info(),
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_impl": ("the reference's codec is CUDA (integration/cuszp_wrapper/"
                           "cuszp_batched_fixed.cu); its C restatement, byte-identical on the "
                           "goldens, on the host cores. The reference's own kernels on the GPU "
                           "are timed in the other arm's reference_kernels object."),
    }


# ---------------------------------------------------------------------------
# Same-run comparison points for the page codec: the reference connector's
# other codecs -- zstd level 1 and LZ4 through the system libraries (as its
# native_lossless.py binds them) and per-page INT8 absmax quantisation
# (vllm_v1_compressed_offload.py:711-724) -- on a bounded sample of pages.


def _load_c_codecs():
    import ctypes.util
    libs = {}
    zpath, lpath = ctypes.util.find_library("zstd"), ctypes.util.find_library("lz4")
    if zpath:
        z = C.CDLL(zpath)
        z.ZSTD_compressBound.argtypes = [C.c_size_t]
        z.ZSTD_compressBound.restype = C.c_size_t
        z.ZSTD_compress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int]
        z.ZSTD_compress.restype = C.c_size_t
        z.ZSTD_decompress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        z.ZSTD_decompress.restype = C.c_size_t
        z.ZSTD_isError.argtypes = [C.c_size_t]
        z.ZSTD_isError.restype = C.c_uint
        libs["zstd1"] = (
            lambda n: int(z.ZSTD_compressBound(n)),
            lambda dst, cap, src, n: int(z.ZSTD_compress(dst, cap, src, n, 1)),
            lambda dst, cap, src, n: int(z.ZSTD_decompress(dst, cap, src, n)))
    if lpath:
        lz = C.CDLL(lpath)
        lz.LZ4_compressBound.argtypes = [C.c_int]
        lz.LZ4_compressBound.restype = C.c_int
        lz.LZ4_compress_default.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int]
        lz.LZ4_compress_default.restype = C.c_int
        lz.LZ4_decompress_safe.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int]
        lz.LZ4_decompress_safe.restype = C.c_int
        libs["lz4"] = (
            lambda n: int(lz.LZ4_compressBound(n)),
            lambda dst, cap, src, n: int(lz.LZ4_compress_default(src, dst, n, cap)),
            lambda dst, cap, src, n: int(lz.LZ4_decompress_safe(src, dst, n, cap)))
    return libs


def codec_baselines(host_pages: torch.Tensor, pages_dev: torch.Tensor, sample: int = 32) -> dict:
    from concurrent.futures import ThreadPoolExecutor
    out = {"sample": f"{sample} pages x {host_pages.shape[1]} BF16 (lossless and CPU INT8); "
                     f"all {pages_dev.shape[0]} pages (GPU INT8)"}
    pages = [np.ascontiguousarray(host_pages[i].view(torch.int16).numpy()) for i in range(sample)]
    raw = sum(p.nbytes for p in pages)
    threads = len(os.sched_getaffinity(0)) or 1
    for name, (bound, comp, decomp) in _load_c_codecs().items():
        cap = bound(pages[0].nbytes)
        bufs = [np.empty(cap, dtype=np.uint8) for _ in pages]
        back = [np.empty_like(p) for p in pages]
        sizes = [0] * len(pages)

        def enc(i):
            sizes[i] = comp(bufs[i].ctypes.data, cap, pages[i].ctypes.data, pages[i].nbytes)

        def dec(i):
            decomp(back[i].ctypes.data, back[i].nbytes, bufs[i].ctypes.data, sizes[i])

        res = {}
        for label, workers in (("1_thread", 1), (f"{threads}_threads", threads)):
            with ThreadPoolExecutor(workers) as pool:
                t0 = time.perf_counter()
                list(pool.map(enc, range(len(pages))))
                t1 = time.perf_counter()
                list(pool.map(dec, range(len(pages))))
                t2 = time.perf_counter()
            res[label] = {"store_gbps": round(raw / (t1 - t0) / 1e9, 3),
                          "restore_gbps": round(raw / (t2 - t1) / 1e9, 3)}
        assert all(np.array_equal(a, b) for a, b in zip(pages, back))
        res["ratio"] = round(raw / sum(sizes), 4)
        out[name] = res

    def int8_store(x):
        f = x.float()
        scale = f.abs().amax(dim=1, keepdim=True) / 127.0
        scale = torch.where(scale == 0, torch.ones_like(scale), scale)
        return torch.clamp(torch.round(f / scale), -127, 127).to(torch.int8), scale

    def int8_restore(q, scale):
        return (q.float() * scale).to(torch.bfloat16)

    cpu = host_pages[:sample]
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    q, sc = int8_store(cpu)
    t1 = time.perf_counter()
    int8_restore(q, sc)
    t2 = time.perf_counter()
    out["int8_cpu_torch"] = {"store_gbps": round(raw / (t1 - t0) / 1e9, 3),
                             "restore_gbps": round(raw / (t2 - t1) / 1e9, 3),
                             "ratio": round(cpu.numel() * 2 / (cpu.numel() + 4 * sample), 4),
                             "threads": threads}
    dev = pages_dev.device
    for _ in range(2):
        qg, sg = int8_store(pages_dev)
        int8_restore(qg, sg)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    e[0].record()
    qg, sg = int8_store(pages_dev)
    e[1].record()
    int8_restore(qg, sg)
    e[2].record()
    torch.cuda.synchronize(dev)
    rawg = pages_dev.numel() * 2
    out["int8_gpu_torch"] = {"store_gbps": round(rawg / (e[0].elapsed_time(e[1]) / 1e3) / 1e9, 1),
                             "restore_gbps": round(rawg / (e[1].elapsed_time(e[2]) / 1e3) / 1e9, 1),
                             "ratio": round(rawg / (pages_dev.numel() + 4 * pages_dev.shape[0]), 4)}
    return out


# ---------------------------------------------------------------------------
# Our arm: libckv through its C ABI.


class OurCodec:
    def __init__(self, device: torch.device, pages_dev: torch.Tensor, chunk_pages: int = 0):
        import _ckv
        self.ckv = _ckv
        self.lib = _ckv.load()
        self.device = device
        cfg = _ckv.Config(EPS, 1, _ckv.DIM_1D, _ckv.MODE_FIXED, _ckv.TYPE_FLOAT)
        self.ctx = C.c_void_p()
        assert self.lib.ckv_create(cfg, device.index, C.byref(self.ctx)) == 0
        self.lib.ckv_set_kernel_timing(self.ctx, 1)
        self.pages = pages_dev
        count, n = pages_dev.shape
        self.count, self.n = count, n
        self.cap = int(self.lib.ckv_estimate_compressed_buffer_size(n * 4))
        self.slab = torch.zeros(count * self.cap, dtype=torch.uint8, device=device)
        self.restored = torch.empty_like(pages_dev)
        self.packed = torch.empty(count * self.cap // 2, dtype=torch.uint8, device=device)
        self.landing = torch.empty_like(self.packed)
        self.pinned = torch.empty(self.packed.numel(), dtype=torch.uint8, pin_memory=True)
        self.in_ptrs = _ckv.ptr_array([pages_dev[i].data_ptr() for i in range(count)])
        self.out_ptrs = _ckv.ptr_array([self.slab.data_ptr() + i * self.cap
                                        for i in range(count)])
        self.dst_ptrs = _ckv.ptr_array([self.restored[i].data_ptr() for i in range(count)])
        self.sizes = (C.c_size_t * count)()
        self.bounds = (C.c_float * count)()
        self.offsets = (C.c_size_t * count)()
        self.total = C.c_size_t(0)
        # store / restore pipeline (ckv_pipe_*): two page-locked host slabs;
        # step k stores into slab k % 2 while restoring step k-1's slab
        # one chunk per job: the codec is ~20x faster than the link, so a
        # store and a restore in flight together keep both directions busy
        # without splitting the job (smaller chunks bound the staging memory)
        self.pipe = C.c_void_p()
        self.chunk = chunk_pages if chunk_pages > 0 else count
        self._check(self.lib.ckv_pipe_create(self.ctx, self.chunk, C.byref(self.pipe)), "pipe")
        host_cap = int(self.lib.ckv_pipe_host_capacity(count, n))
        self.hslab = [torch.empty(host_cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.hmeta = [{"offsets": (C.c_size_t * count)(), "sizes": (C.c_size_t * count)(),
                       "bounds": (C.c_float * count)(), "total": C.c_size_t(0)} for _ in range(2)]
        self.restored_e2e = torch.empty_like(pages_dev)
        self.dst_e2e = _ckv.ptr_array([self.restored_e2e[i].data_ptr() for i in range(count)])
        self.e2e_k = 0
        self.t_store = 0
        self.t_restore = 0
        self.side = torch.cuda.Stream(device)
        self.cont_pages = None
        self.cont_ptrs = None
        self._stream = None
        self.slab_set = [0, 0]   # which copy of the pages each host slab holds

    def _check(self, status: int, what: str):
        if status != 0:
            raise RuntimeError(f"{what}: {self.ckv.error_message(self.lib, self.ctx, status)}")

    def stream(self) -> int:
        """The CUDA stream the calls run on (the device's current stream, as a
        serving engine keeps its handle rather than looking it up per call)."""
        if self._stream is None:
            self._stream = torch.cuda.current_stream(self.device).cuda_stream
        return self._stream

    def store(self):
        self._check(self.lib.ckv_compress_batch_fixed_bf16(
            self.ctx, self.in_ptrs, self.out_ptrs, None, self.count, self.n, self.cap,
            self.sizes, self.bounds, self.stream()), "compress")

    def restore(self, ins=None):
        self._check(self.lib.ckv_decompress_batch_fixed_bf16_scatter(
            self.ctx, ins if ins is not None else self.out_ptrs, self.sizes, self.count,
            self.dst_ptrs, self.count, self.n, 1, self.n, self.bounds, self.stream()),
            "decompress")

    def step(self):
        self.store()
        self.restore()

    def step_e2e(self):
        self.store()
        self._check(self.lib.ckv_pack(self.ctx, self.out_ptrs, self.sizes, self.count,
                                      self.packed.data_ptr(), self.packed.numel(), 16,
                                      self.offsets, C.byref(self.total), self.stream()),
                    "pack")
        total = self.total.value
        self.pinned[:total].copy_(self.packed[:total], non_blocking=True)
        self.landing[:total].copy_(self.pinned[:total], non_blocking=True)
        base = self.landing.data_ptr()
        ins = self.ckv.ptr_array([base + o for o in self.offsets])
        self.restore(ins)
        return total

    def e2e_sets(self):
        """The pages and two rotations of them (same pages, other addresses):
        steps that cycle through the three read 352 MB of inputs, more than
        L2 holds, so back-to-back steps need no flush between them."""
        if self.cont_ptrs is None:
            self.cont_pages = [self.pages] + [self.pages.roll(i, 0).contiguous() for i in (1, 2)]
            self.cont_ptrs = [self.ckv.ptr_array([p[i].data_ptr() for i in range(self.count)])
                              for p in self.cont_pages]
        return self.cont_ptrs

    def step_e2e_pipelined(self, pages_set=None, join=True):
        """Store this step's pages into one host slab while the previous
        step's slab is restored: both directions of the link at once.
        join=False leaves the step's work in flight (the next step's calls
        are ordered after it on the device by the pipeline's tickets)."""
        in_ptrs = self.in_ptrs if pages_set is None else self.e2e_sets()[pages_set]
        k = self.e2e_k
        self.e2e_k += 1
        main = torch.cuda.current_stream(self.device)
        a, b = self.hmeta[k % 2], self.hmeta[(k + 1) % 2]
        prev_restore = self.t_restore   # the last reader of slab k % 2
        restored = 0
        if k > 0:
            # queued first, on a side stream: the restore never blocks the
            # host, so its copies start while the store below is being queued
            self.side.wait_stream(main)
            t_rest = C.c_uint64(0)
            self._check(self.lib.ckv_pipe_restore_bf16(
                self.pipe, self.hslab[(k + 1) % 2].data_ptr(), b["offsets"], b["sizes"],
                b["bounds"], self.count, self.n, self.dst_e2e, self.t_store, C.byref(t_rest),
                self.side.cuda_stream), "pipe restore")
            self.t_restore = t_rest.value
            restored = b["total"].value
        t_store = C.c_uint64(0)
        self._check(self.lib.ckv_pipe_store_bf16(
            self.pipe, in_ptrs, None, self.count, self.n, self.hslab[k % 2].data_ptr(),
            self.hslab[k % 2].numel(), a["offsets"], a["sizes"], a["bounds"],
            C.byref(a["total"]), prev_restore, C.byref(t_store), main.cuda_stream), "pipe store")
        self.t_store = t_store.value
        self.slab_set[k % 2] = pages_set or 0
        if join:
            self.finish_e2e()
        return a["total"].value, restored

    def finish_e2e(self):
        """The caller's stream waits for the last store and restore."""
        main = torch.cuda.current_stream(self.device)
        self._check(self.lib.ckv_pipe_join(self.pipe, self.t_store, main.cuda_stream),
                    "pipe join")
        main.wait_stream(self.side)

    def e2e_continuous(self, steps: int, warmup: int = 3):
        """`steps` pipelined steps back to back, as a serving engine offloads
        and reloads continuously: no synchronisation between steps, inputs
        cycling through the three copies of the pages.  Device time from
        before the first call to the join after the last (seconds), and the
        steps' (stored, restored) byte counts."""
        main = torch.cuda.current_stream(self.device)
        self.e2e_sets()
        for i in range(warmup):
            self.step_e2e_pipelined(pages_set=i % 3, join=False)
        self.finish_e2e()
        torch.cuda.synchronize(self.device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        collect = gc.isenabled()
        gc.disable()
        try:
            start.record(main)
            totals = [self.step_e2e_pipelined(pages_set=i % 3, join=False) for i in range(steps)]
            self.finish_e2e()
            end.record(main)
            end.synchronize()
        finally:
            if collect:
                gc.enable()
        return start.elapsed_time(end) / 1e3, totals

    def run_continuous(self, step, steps: int, warmup: int = 3) -> float:
        """step(i) for `steps` steps back to back (no synchronisation between
        them), joined at the end: device seconds."""
        main = torch.cuda.current_stream(self.device)
        for i in range(warmup):
            step(i)
        self.finish_e2e()
        torch.cuda.synchronize(self.device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        collect = gc.isenabled()
        gc.disable()
        try:
            start.record(main)
            for i in range(steps):
                step(i)
            self.finish_e2e()
            end.record(main)
            end.synchronize()
        finally:
            if collect:
                gc.enable()
        return start.elapsed_time(end) / 1e3

    def e2e_continuous_matches(self) -> bool:
        """The last restore of e2e_continuous decoded the slab stored one step
        before the last, which held copy j of the pages: bit for bit the
        kernel path's restore of the same pages, rotated by j."""
        torch.cuda.synchronize(self.device)
        j = self.slab_set[(self.e2e_k - 2) % 2]
        want = self.restored.roll(j, 0)
        return bool(torch.equal(self.restored_e2e.view(torch.int16), want.view(torch.int16)))

    def step_store_only(self, pages_set=None, join=True):
        """One direction alone: every page stored into host slab 0 (device to
        host), nothing else on the link."""
        main = torch.cuda.current_stream(self.device)
        in_ptrs = self.in_ptrs if pages_set is None else self.e2e_sets()[pages_set]
        a = self.hmeta[0]
        t_store = C.c_uint64(0)
        self._check(self.lib.ckv_pipe_store_bf16(
            self.pipe, in_ptrs, None, self.count, self.n, self.hslab[0].data_ptr(),
            self.hslab[0].numel(), a["offsets"], a["sizes"], a["bounds"], C.byref(a["total"]),
            self.t_restore, C.byref(t_store), main.cuda_stream), "pipe store")
        self.t_store = t_store.value
        if join:
            self._check(self.lib.ckv_pipe_join(self.pipe, self.t_store, main.cuda_stream),
                        "pipe join")
        return a["total"].value

    def step_restore_only(self):
        """The other direction alone: host slab 0 restored into the pages."""
        main = torch.cuda.current_stream(self.device)
        a = self.hmeta[0]
        t_rest = C.c_uint64(0)
        self._check(self.lib.ckv_pipe_restore_bf16(
            self.pipe, self.hslab[0].data_ptr(), a["offsets"], a["sizes"], a["bounds"], self.count,
            self.n, self.dst_e2e, self.t_store, C.byref(t_rest), main.cuda_stream), "pipe restore")
        self.t_restore = t_rest.value
        return a["total"].value

    def e2e_matches(self) -> bool:
        torch.cuda.synchronize(self.device)
        return bool(torch.equal(self.restored_e2e.view(torch.int16), self.restored.view(torch.int16)))

    def kernel_ms(self, kind: int) -> float:
        ms = C.c_float(0.0)
        self._check(self.lib.ckv_kernel_time(self.ctx, kind, C.byref(ms)), "kernel time")
        return float(ms.value)

    def launches(self) -> int:
        return int(self.lib.ckv_kernel_launches())

    def compressed_bytes(self) -> int:
        return int(sum(self.sizes))

    def verify(self) -> bool:
        """Round-trip check of the last restore against the pages."""
        torch.cuda.synchronize(self.device)
        b = torch.tensor(list(self.bounds), device=self.device).view(-1, 1)
        x, xh = self.pages.float(), self.restored.float()
        return bool(((x - xh).abs() <= b * 1.01 + 1e-7 + x.abs() * 2.0 ** -8).all())


class RefCodec:
    """The reference's kernels (oracle/_ref) driven like CuSZpWrapper."""

    def __init__(self, device: torch.device, pages_dev: torch.Tensor):
        from oracle.oracle import RefKernels
        self.ref = RefKernels()
        self.device = device
        self.pages = pages_dev
        count, n = pages_dev.shape
        self.count, self.n = count, n
        self.cap = 8 * n
        self.slab = torch.zeros(count * self.cap, dtype=torch.uint8, device=device)
        self.restored = torch.empty_like(pages_dev)
        self.in_ptrs = [pages_dev[i].data_ptr() for i in range(count)]
        self.out_ptrs = [self.slab.data_ptr() + i * self.cap for i in range(count)]
        self.dst_ptrs = [self.restored[i].data_ptr() for i in range(count)]
        self.pinned = torch.empty(count * self.cap // 2, dtype=torch.uint8, pin_memory=True)
        self.landing = torch.empty(count * self.cap // 2, dtype=torch.uint8, device=device)
        self.sizes = None
        self.bounds = None

    def stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def store(self):
        self.sizes, self.bounds = self.ref.compress(
            self.in_ptrs, self.out_ptrs, self.cap, self.n, [EPS] * self.count, relative=True,
            stream=self.stream(), zero_outputs=False)

    def restore(self, ins=None):
        self.ref.decompress(ins or self.out_ptrs, self.n, self.bounds, 1, self.dst_ptrs,
                            per_page=1, elements_per_dest=self.n, stream=self.stream())

    def step(self):
        self.store()
        self.restore()

    def step_e2e(self):
        # vllm_v1_compressed_offload.py:371-447 (torch.cat into a GPU slab, one
        # D2H) and :1618-1711 (one H2D, batched decode from the slab).
        self.store()
        views, offsets, pos = [], [], 0
        for i in range(self.count):
            start = (pos + 7) // 8 * 8
            if start > pos:
                views.append(self.landing[:start - pos])
            size = int(self.sizes[i])
            views.append(self.slab[i * self.cap:i * self.cap + size])
            offsets.append(start)
            pos = start + size
        packed = torch.cat(views)
        self.pinned[:pos].copy_(packed, non_blocking=True)
        self.landing[:pos].copy_(self.pinned[:pos], non_blocking=True)
        base = self.landing.data_ptr()
        self.restore([base + o for o in offsets])
        return pos

    def kernel_ms(self, kind):
        return None

    def launches(self):
        return 0

    def compressed_bytes(self):
        return int(sum(int(s) for s in self.sizes))

    def verify(self) -> bool:
        torch.cuda.synchronize(self.device)
        b = torch.tensor(list(self.bounds), device=self.device).view(-1, 1)
        x, xh = self.pages.float(), self.restored.float()
        return bool(((x - xh).abs() <= b * 1.01 + 1e-7 + x.abs() * 2.0 ** -8).all())


# ---------------------------------------------------------------------------


def timed_steps(fn, steps: int, flush: torch.Tensor, device, after=None):
    """Per-step CUDA-event times (ms) and fn's results; L2 flushed before
    every step, outside the timed events.  The collector is paused meanwhile:
    a collection between the compress call's return and the decompress
    launch would stall the device for its whole length."""
    stream = torch.cuda.current_stream(device)
    times, results = [], []
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
    collect = gc.isenabled()
    gc.disable()
    try:
        for start, end in events:
            flush.zero_()
            start.record(stream)
            results.append(fn())
            end.record(stream)
            end.synchronize()
            if after is not None:
                after()
    finally:
        if collect:
            gc.enable()
    times = [start.elapsed_time(end) for start, end in events]
    return times, results


def pipeline_codecs(codec, steps: int, flush: torch.Tensor, device) -> dict:
    """The reference's INT8 and raw encodings (vllm_v1_compressed_offload.py:
    711-724 / :2090-2116 and :1578-1615) through the same store / restore
    pipeline, timed like the fixed-mode e2e: step k stores the pages into one
    page-locked slab while step k-1's slab is restored, both on the device
    clock.  Restores are checked against the reference's torch expression
    (INT8) or the pages themselves (raw)."""
    lib, ck = codec.lib, codec.ckv
    count, n = codec.count, codec.n
    page_bytes = n * 2
    raw_bytes = count * page_bytes
    x = codec.pages.float()
    scale = x.abs().amax(dim=1, keepdim=True) / 127.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.clamp(torch.round(x / scale), -127, 127).to(torch.int8)   # -0 becomes 0 here
    want_int8 = (q.to(torch.float32) * scale).to(torch.bfloat16)
    del q
    del x
    out = {}
    for name in ("int8", "raw"):
        cap = int(lib.ckv_pipe_host_capacity_int8(count, n) if name == "int8"
                  else lib.ckv_pipe_host_capacity_raw(count, page_bytes))
        slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * count)(), "s": (C.c_size_t * count)(), "t": C.c_size_t(0)}
                for _ in range(2)]
        dst = torch.empty_like(codec.pages)
        dptr = ck.ptr_array([dst[i].data_ptr() for i in range(count)])
        side = torch.cuda.Stream(device)
        state = {"k": 0, "ts": 0, "tr": 0}

        def step():
            k = state["k"]
            state["k"] += 1
            main = torch.cuda.current_stream(device)
            a, b = meta[k % 2], meta[(k + 1) % 2]
            prev_restore = state["tr"]
            restored = 0
            if k > 0:
                side.wait_stream(main)
                tr = C.c_uint64(0)
                slab = slabs[(k + 1) % 2].data_ptr()
                if name == "int8":
                    st = lib.ckv_pipe_restore_int8(codec.pipe, slab, b["o"], count, n, dptr,
                                                   state["ts"], C.byref(tr), side.cuda_stream)
                else:
                    st = lib.ckv_pipe_restore_raw(codec.pipe, slab, b["o"], count, page_bytes, dptr,
                                                  state["ts"], C.byref(tr), side.cuda_stream)
                codec._check(st, f"{name} pipe restore")
                state["tr"] = tr.value
                restored = b["t"].value
            ts = C.c_uint64(0)
            slab = slabs[k % 2].data_ptr()
            if name == "int8":
                st = lib.ckv_pipe_store_int8(codec.pipe, codec.in_ptrs, count, n, slab, cap, a["o"],
                                             a["s"], C.byref(a["t"]), prev_restore, C.byref(ts),
                                             main.cuda_stream)
            else:
                st = lib.ckv_pipe_store_raw(codec.pipe, codec.in_ptrs, count, page_bytes, slab, cap,
                                            a["o"], C.byref(a["t"]), prev_restore, C.byref(ts),
                                            main.cuda_stream)
            codec._check(st, f"{name} pipe store")
            state["ts"] = ts.value
            codec._check(lib.ckv_pipe_join(codec.pipe, state["ts"], main.cuda_stream), "pipe join")
            main.wait_stream(side)
            return a["t"].value, restored

        for _ in range(3):
            step()
        times, totals = timed_steps(step, steps, flush, device)
        torch.cuda.synchronize(device)
        ok = bool(torch.equal(dst.view(torch.int16),
                              (want_int8 if name == "int8" else codec.pages).view(torch.int16)))
        stored = totals[-1][0]
        ms = [C.c_float(0.0) for _ in range(2)]
        kinds = (3, 4) if name == "int8" else (5, 5)
        for m, kind in zip(ms, kinds):
            codec._check(lib.ckv_kernel_time(codec.ctx, kind, C.byref(m)), "kernel time")
        t = sum(times) / 1e3
        out[name] = {
            "e2e_gbps": round(job_rate(1, raw_bytes, steps, t), 3),
            "ms_per_step": round(t * 1e3 / steps, 4),
            "compression_ratio": round(raw_bytes / stored, 4),
            "d2h_bytes_per_step": int(stored), "h2d_bytes_per_step": int(totals[-1][1]),
            "restore_ok": ok,
            "store_kernel_ms": round(ms[0].value, 4),
            "restore_kernel_ms": round(ms[1].value, 4) if name == "int8" else None,
            "path": f"ckv_pipe_store_{name} overlapped with ckv_pipe_restore_{name} of the "
                    "previous step's slab, one chunk per job",
        }
    return out


def c1_leg(codec, steps: int, flush: torch.Tensor, device) -> dict:
    """C1: one layer's K and V of 64 pages, 8192
    BF16 each (K, V ~ N(0,1) x LogNormal(0, 0.5) per (head, channel),
    seeded), REL 1e-4, compressed and decompressed through the C ABI; and
    the same pages zero-padded to 36864 elements, the unit the reference's
    connector would compress (vllm_v1_compressed_offload.py:49, 904-909)."""
    lib, ck = codec.lib, codec.ckv
    g = torch.Generator().manual_seed(0)
    scale = torch.empty(2, HEADS, HEAD_DIM).log_normal_(0.0, 0.5, generator=g)
    x = torch.randn(64, 2, TOKENS, HEADS, HEAD_DIM, generator=g) * scale[None, :, None, :, :]
    pages8k = x.to(torch.bfloat16).view(64, -1).to(device)
    out = {}
    for label, n in (("n8192", 8192), ("padded36864", 36864)):
        pages = torch.zeros(64, n, dtype=torch.bfloat16, device=device)
        pages[:, :8192] = pages8k
        cap = int(lib.ckv_estimate_compressed_buffer_size(n * 4))
        slab = torch.zeros(64 * cap, dtype=torch.uint8, device=device)
        restored = torch.zeros_like(pages)
        ins = ck.ptr_array([pages[i].data_ptr() for i in range(64)])
        outs = ck.ptr_array([slab.data_ptr() + i * cap for i in range(64)])
        dsts = ck.ptr_array([restored[i].data_ptr() for i in range(64)])
        eps = (C.c_float * 64)(*([1e-4] * 64))
        sizes, bounds = (C.c_size_t * 64)(), (C.c_float * 64)()
        s = torch.cuda.current_stream(device).cuda_stream
        enc_ms, dec_ms = [], []

        def step():
            codec._check(lib.ckv_compress_batch_fixed_bf16(codec.ctx, ins, outs, eps, 64, n, cap,
                                                           sizes, bounds, s), "c1 compress")
            codec._check(lib.ckv_decompress_batch_fixed_bf16_scatter(
                codec.ctx, outs, sizes, 64, dsts, 64, n, 1, n, bounds, s), "c1 decompress")

        def kernel_times():
            enc_ms.append(codec.kernel_ms(0))
            dec_ms.append(codec.kernel_ms(1))

        for _ in range(3):
            step()
        times, _ = timed_steps(step, steps, flush, device, after=kernel_times)
        torch.cuda.synchronize(device)
        raw = 64 * n * 2
        comp = int(sum(sizes))
        b = torch.tensor(list(bounds), device=device).view(-1, 1)
        ok = bool(((pages.float() - restored.float()).abs() <=
                   b * 1.01 + 1e-7 + pages.float().abs() * 2.0 ** -8).all())
        enc, dec = statistics.mean(enc_ms) / 1e3, statistics.mean(dec_ms) / 1e3
        out[label] = {
            "value_gbps": round(job_rate(1, raw, steps, sum(times) / 1e3), 3),
            "compression_ratio": round(raw / comp, 4),
            "ratio_of_the_8192_elements": round(64 * 8192 * 2 / comp, 4),
            "encode_ms": round(enc * 1e3, 4), "decode_ms": round(dec * 1e3, 4),
            "encode_gbps": round((raw + comp) / enc / 1e9, 2),
            "decode_gbps": round((raw + comp) / dec / 1e9, 2),
            "round_trip_ok": ok,
        }
    out["workload"] = ("C1: 64 pages x [K,V][16 tokens][2 heads][128] = 8192 BF16, REL 1e-4, "
                       "compress + decompress per step (1 MiB); L2 flushed between steps")
    return out


def pipe_pages_leg(codec, pages: torch.Tensor, eps: float, steps: int, flush: torch.Tensor,
                   device) -> dict:
    """Uniform pages through the store / restore pipeline (one chunk per call):
    the store alone, the restore alone, a store overlapped with the restore of
    the previous step's slab, and raw pinned copies of the same bytes one way
    at a time; the restore is checked against the pages' bounds."""
    lib, ck = codec.lib, codec.ckv
    count, n = pages.shape
    raw = count * n * 2
    pipe = C.c_void_p()
    codec._check(lib.ckv_pipe_create(codec.ctx, count, C.byref(pipe)), "pipe")
    try:
        cap = int(lib.ckv_pipe_host_capacity(count, n))
        slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * count)(), "s": (C.c_size_t * count)(),
                 "b": (C.c_float * count)(), "t": C.c_size_t(0)} for _ in range(2)]
        dst = torch.zeros_like(pages)
        src = ck.ptr_array([pages[i].data_ptr() for i in range(count)])
        dptr = ck.ptr_array([dst[i].data_ptr() for i in range(count)])
        epsa = (C.c_float * count)(*([eps] * count))
        side = torch.cuda.Stream(device)
        st = {"k": 0, "ts": 0, "tr": 0}

        def store(k, stream):
            a = meta[k]
            t = C.c_uint64(0)
            codec._check(lib.ckv_pipe_store_bf16(
                pipe, src, epsa, count, n, slabs[k].data_ptr(), cap, a["o"], a["s"], a["b"],
                C.byref(a["t"]), st["tr"], C.byref(t), stream), "pipe store")
            st["ts"] = t.value
            return a["t"].value

        def restore(k, stream):
            b = meta[k]
            t = C.c_uint64(0)
            codec._check(lib.ckv_pipe_restore_bf16(
                pipe, slabs[k].data_ptr(), b["o"], b["s"], b["b"], count, n, dptr, st["ts"],
                C.byref(t), stream), "pipe restore")
            st["tr"] = t.value
            return b["t"].value

        def store_only():
            main = torch.cuda.current_stream(device)
            moved = store(0, main.cuda_stream)
            codec._check(lib.ckv_pipe_join(pipe, st["ts"], main.cuda_stream), "join")
            return moved

        def restore_only():
            return restore(0, torch.cuda.current_stream(device).cuda_stream)

        def overlapped():
            k = st["k"]
            st["k"] += 1
            main = torch.cuda.current_stream(device)
            if k > 0:
                side.wait_stream(main)
                restore((k + 1) % 2, side.cuda_stream)
            moved = store(k % 2, main.cuda_stream)
            codec._check(lib.ckv_pipe_join(pipe, st["ts"], main.cuda_stream), "join")
            main.wait_stream(side)
            return moved

        for fn in (store_only, restore_only):
            for _ in range(3):
                fn()
        t_st, moved = timed_steps(store_only, steps, flush, device)
        t_rs, _ = timed_steps(restore_only, steps, flush, device)
        torch.cuda.synchronize(device)
        b = torch.tensor(list(meta[0]["b"]), device=device).view(-1, 1)
        ok = bool(((pages.float() - dst.float()).abs() <=
                   b * 1.01 + 1e-7 + pages.float().abs() * 2.0 ** -8).all())
        for _ in range(3):
            overlapped()
        t_ov, _ = timed_steps(overlapped, steps, flush, device)
        t_d2h, t_h2d = raw_one_way(pages, steps, flush, device)
        out = direction_fields(1, raw, steps, sum(t_st) / 1e3, sum(t_rs) / 1e3, raw, steps,
                               t_d2h, t_h2d)
        out.update({
            "overlapped_gbps": round(job_rate(1, raw, steps, sum(t_ov) / 1e3), 3),
            "ms_store": round(sum(t_st) / steps, 4), "ms_restore": round(sum(t_rs) / steps, 4),
            "compression_ratio": round(raw / max(1, moved[-1]), 4),
            "d2h_bytes_per_store": int(moved[-1]), "restore_ok": ok,
        })
        return out
    finally:
        torch.cuda.synchronize(device)
        lib.ckv_pipe_destroy(pipe)


def c1_pipeline(codec, steps: int, flush: torch.Tensor, device, batches=(1, 16)) -> dict:
    """C1 with host copies: jobs of 64 one-layer units (8192 BF16 each, 1 MiB)
    through the pipeline, one job per call and `batch` jobs per call (the
    units of several jobs in one encode and one decode launch)."""
    g = torch.Generator().manual_seed(0)
    scale = torch.empty(2, HEADS, HEAD_DIM).log_normal_(0.0, 0.5, generator=g)
    x = torch.randn(64, 2, TOKENS, HEADS, HEAD_DIM, generator=g) * scale[None, :, None, :, :]
    job = x.to(torch.bfloat16).view(64, -1).to(device)
    out = {"workload": "C1 with host copies: jobs of 64 units x 8192 BF16 (1 MiB), REL 1e-4, "
                       "through ckv_pipe_store_bf16 / ckv_pipe_restore_bf16"}
    for batch in batches:
        out[f"jobs_per_call_{batch}"] = pipe_pages_leg(codec, job.repeat(batch, 1), 1e-4, steps,
                                                       flush, device)
    return out


class _BlockSpec:
    """A transfer spec as vLLM's GPULoadStoreSpec / CPULoadStoreSpec present
    it to a handler: its block ids."""

    def __init__(self, ids):
        self.block_ids = np.asarray(ids, dtype=np.int64)


def plugin_api_leg(codec, steps: int, flush: torch.Tensor, device) -> dict:
    """The connector-facing API timed on the C2 pages: kv_offload's
    CompressedCpuGpuOffloadingHandlers (vLLM's OffloadingHandler interface,
    vllm_v1_compressed_offload.py:2365-2470) -- transfer_async of a store job
    (GPU blocks -> CPU blocks) and of a load job (CPU blocks -> other GPU
    blocks), each waited for with the handler's wait() -- next to the same
    jobs through the C ABI (ckv_pipe_store_bf16 / ckv_pipe_restore_bf16 +
    ckv_pipe_wait).  Both on the host clock (call to completion); the gap is
    what the job layer (job header, slab pool, Python) costs."""
    import kv_offload as ko
    lib = codec.lib
    count, n = codec.count, codec.n
    raw = count * n * 2
    kv = torch.empty(2 * count, n, dtype=torch.bfloat16, device=device)
    kv[:count] = codec.pages
    h = ko.CompressedCpuGpuOffloadingHandlers(kv, error_bound=EPS, device_id=device.index,
                                              chunk_pages=count)
    try:
        gpu_src = _BlockSpec(range(count))
        gpu_dst = _BlockSpec(range(count, 2 * count))
        cpu = [_BlockSpec(range(count)), _BlockSpec(range(count, 2 * count))]
        job = [0]

        def timed(fn) -> float:
            flush.zero_()
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            fn()
            return time.perf_counter() - t0

        def store(c):
            job[0] += 1
            assert h.gpu_to_cpu_handler.transfer_async(job[0], (gpu_src, cpu[c]))
            return job[0]

        def load(c):
            job[0] += 1
            assert h.cpu_to_gpu_handler.transfer_async(job[0], (cpu[c], gpu_dst))
            return job[0]

        def store_wait():
            h.gpu_to_cpu_handler.wait({store(0)})

        def load_wait():
            h.cpu_to_gpu_handler.wait({load(0)})

        state = {"k": 0}

        def overlapped():
            k = state["k"]
            state["k"] += 1
            ld = load((k + 1) % 2) if k > 0 else None
            st = store(k % 2)
            h.gpu_to_cpu_handler.wait({st})
            if ld is not None:
                h.cpu_to_gpu_handler.wait({ld})

        collect = gc.isenabled()
        gc.disable()
        try:
            for fn in (store_wait, load_wait, overlapped, overlapped, overlapped):
                fn()
            t_store = sum(timed(store_wait) for _ in range(steps))
            t_load = sum(timed(load_wait) for _ in range(steps))
            t_ov = sum(timed(overlapped) for _ in range(steps))
            # the same jobs through the C ABI, host clock
            a = codec.hmeta[0]
            tick = C.c_uint64(0)

            def abi_store():
                codec._check(lib.ckv_pipe_store_bf16(
                    codec.pipe, codec.in_ptrs, None, count, n, codec.hslab[0].data_ptr(),
                    codec.hslab[0].numel(), a["offsets"], a["sizes"], a["bounds"],
                    C.byref(a["total"]), codec.t_restore, C.byref(tick),
                    torch.cuda.current_stream(device).cuda_stream), "pipe store")
                codec.t_store = tick.value
                codec._check(lib.ckv_pipe_wait(codec.pipe, codec.t_store), "pipe wait")

            def abi_restore():
                codec._check(lib.ckv_pipe_restore_bf16(
                    codec.pipe, codec.hslab[0].data_ptr(), a["offsets"], a["sizes"], a["bounds"],
                    count, n, codec.dst_e2e, codec.t_store, C.byref(tick),
                    torch.cuda.current_stream(device).cuda_stream), "pipe restore")
                codec.t_restore = tick.value
                codec._check(lib.ckv_pipe_wait(codec.pipe, codec.t_restore), "pipe wait")

            abi_store()
            abi_restore()
            t_abi_store = sum(timed(abi_store) for _ in range(steps))
            t_abi_restore = sum(timed(abi_restore) for _ in range(steps))
        finally:
            if collect:
                gc.enable()
        torch.cuda.synchronize(device)
        ok = bool(torch.equal(kv[count:].view(torch.int16), codec.restored.view(torch.int16)))
        g = lambda t: round(raw * steps / t / 1e9, 3)   # noqa: E731
        return {
            "workload": "C2 pages through kv_offload.CompressedCpuGpuOffloadingHandlers "
                        "(transfer_async + wait), host clock",
            "store_gbps": g(t_store), "restore_gbps": g(t_load),
            "overlapped_gbps": round(2 * raw * steps / t_ov / 1e9, 3),
            "c_abi_store_gbps": g(t_abi_store), "c_abi_restore_gbps": g(t_abi_restore),
            "handler_vs_c_abi_store": round(t_abi_store / t_store, 4),
            "handler_vs_c_abi_restore": round(t_abi_restore / t_load, 4),
            "restore_matches_kernel_path": ok,
        }
    finally:
        h.shutdown()
        del kv


def compare_with_reference(codec, ref) -> dict:
    """Our compressed pages against the reference kernels' on the same pages
    and bounds: sizes, resolved bounds (bit for bit), the bytes the reference
    defines (rate bytes of real blocks, [0, ceil(n/32)), and the payload,
    [G*1024, size)), and the BF16 each decoder writes into zeroed pages."""
    n, count = codec.n, codec.count
    nb = (n + 31) // 32
    hdr = (n + 32767) // 32768 * 1024
    sizes_ok = [int(a) for a in codec.sizes] == [int(b) for b in ref.sizes]
    bounds_ok = bool(np.array_equal(np.ctypeslib.as_array(codec.bounds).view(np.uint32),
                                    np.asarray(ref.bounds, dtype=np.float32).view(np.uint32)))
    ours = codec.slab.view(count, codec.cap)
    theirs = ref.slab.view(count, ref.cap)
    bytes_ok = sizes_ok and bool(torch.equal(ours[:, :nb], theirs[:, :nb]))
    if bytes_ok:
        for i in range(count):
            size = int(codec.sizes[i])
            if not torch.equal(ours[i, hdr:size], theirs[i, hdr:size]):
                bytes_ok = False
                break
    codec.restored.zero_()
    ref.restored.zero_()
    codec.restore()
    ref.restore()
    torch.cuda.synchronize(codec.device)
    decoded_ok = bool(torch.equal(codec.restored.view(torch.int16), ref.restored.view(torch.int16)))
    return {"pages": count, "sizes_match": sizes_ok, "bounds_match": bounds_ok,
            "bytes_match": bytes_ok, "decoded_match": decoded_ok}


def reference_kernels_leg(device, pages_dev: torch.Tensor, steps: int, warmup: int,
                          flush: torch.Tensor, codec=None) -> dict | None:
    """The reference's own kernels on the same GPU and pages: its batched BF16
    kernels (integration/cuszp_wrapper/cuszp_batched_fixed.cu, built unchanged
    in oracle/_ref) driven as CuSZpWrapper drives them, and its connector's
    store / restore (torch.cat packing, one D2H, one H2D, batched scatter
    decode) for the end-to-end number."""
    from oracle import build as oracle_build
    if not oracle_build.REF_SO.exists():
        return None
    ref = RefCodec(device, pages_dev)
    for _ in range(warmup):
        ref.step()
        ref.step_e2e()
    torch.cuda.synchronize(device)
    raw = pages_dev.numel() * 2
    v_ms, _ = timed_steps(ref.step, steps, flush, device)
    e_ms, totals = timed_steps(ref.step_e2e, steps, flush, device)
    ok = ref.verify()
    parity = None
    if codec is not None:
        ref.step()
        codec.store()
        parity = compare_with_reference(codec, ref)
    return {
        "parity_with_ours": parity,
        "value": round(job_rate(1, raw, steps, sum(v_ms) / 1e3), 3),
        "ms_per_step": round(sum(v_ms) / steps, 4),
        "e2e": round(job_rate(1, raw, steps, sum(e_ms) / 1e3), 3),
        "e2e_ms_per_step": round(sum(e_ms) / steps, 4),
        "h2d_bytes_per_step": int(totals[-1]), "d2h_bytes_per_step": int(totals[-1]),
        "compression_ratio": round(raw / ref.compressed_bytes(), 4),
        "restore_ok": ok,
        "path": "the reference's batched BF16 kernels (oracle/_ref, built unchanged from "
                "integration/cuszp_wrapper/cuszp_batched_fixed.cu) driven like CuSZpWrapper; "
                "e2e: compress, torch.cat pack, one D2H, one H2D, decompress",
    }


C3_LOW_LAYERS = (0, 1, 2, 5, 19, 20, 21)   # 1e-5; the other 21 layers at 1e-4


def c3_host_slabs(codec, repeat: int = 8) -> list[torch.Tensor]:
    """The C3 leg's two page-locked slabs, allocated before the other legs'
    (page-locked buffers allocated late in the run measured slower copies)."""
    lib = codec.lib
    prefix, layers = 2, LAYERS
    epl = codec.n // (prefix * layers)
    high = [i for i in range(layers) if i not in C3_LOW_LAYERS]
    sel = (C.c_size_t * 2)(len(C3_LOW_LAYERS), len(high))
    cap = int(lib.ckv_pipe_host_capacity_groups(codec.count * repeat, sel, 2, prefix, epl))
    import kv_offload as ko
    slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    ko.prefault_pinned(slabs, codec.device)   # first use at full speed, no untimed pass
    return slabs


def layer_groups_c3(codec, steps: int, flush: torch.Tensor, device, repeat: int = 8,
                    chunk_pages: int = 0, slabs=None) -> dict:
    """C3: the mixed per-layer profile (7 layers at 1e-5, 21 at 1e-4, the
    reference's calibrated assignment) over 2048 pages, each page stored as
    two layer segments (ckv_pipe_store_bf16_groups) while the previous
    step's slab is restored into all 28 layers (ckv_pipe_restore_bf16_groups),
    timed like the fixed-mode e2e.  The 2048 pages are the C2 pages repeated
    `repeat` times on the device.  The restore is checked per element against
    its segment's bound."""
    lib, ck = codec.lib, codec.ckv
    prefix, layers = 2, LAYERS
    epl = codec.n // (prefix * layers)
    high = tuple(i for i in range(layers) if i not in C3_LOW_LAYERS)
    groups = [(1e-5, C3_LOW_LAYERS), (1e-4, high)]          # ascending bound
    G = len(groups)
    pages = codec.pages.repeat(repeat, 1)
    count = pages.shape[0]
    raw_bytes = count * codec.n * 2
    index = [torch.tensor(sel, dtype=torch.int64, device=device) for _b, sel in groups]
    idx = (C.c_void_p * G)(*[t.data_ptr() for t in index])
    sel = (C.c_size_t * G)(*[len(s) for _b, s in groups])
    eps = (C.c_float * G)(*[b for b, _s in groups])
    pipe = C.c_void_p()
    codec._check(lib.ckv_pipe_create(codec.ctx, chunk_pages or count, C.byref(pipe)), "c3 pipe")
    try:
        cap = int(lib.ckv_pipe_host_capacity_groups(count, sel, G, prefix, epl))
        if slabs is None or min(t.numel() for t in slabs) < cap:
            slabs = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * (count * G))(), "s": (C.c_size_t * (count * G))(),
                 "b": (C.c_float * (count * G))(), "t": C.c_size_t(0)} for _ in range(2)]
        dst = torch.zeros_like(pages)
        src_ptrs = ck.ptr_array([pages[i].data_ptr() for i in range(count)])
        dptr = ck.ptr_array([dst[i].data_ptr() for i in range(count)])
        side = torch.cuda.Stream(device)
        state = {"k": 0, "ts": 0, "tr": 0}

        def step():
            k = state["k"]
            state["k"] += 1
            main = torch.cuda.current_stream(device)
            a, b = meta[k % 2], meta[(k + 1) % 2]
            prev_restore = state["tr"]
            restored = 0
            if k > 0:
                side.wait_stream(main)
                tr = C.c_uint64(0)
                codec._check(lib.ckv_pipe_restore_bf16_groups(
                    pipe, slabs[(k + 1) % 2].data_ptr(), b["o"], b["s"], b["b"], count, idx, sel,
                    G, prefix, layers, epl, dptr, state["ts"], C.byref(tr), side.cuda_stream),
                    "c3 restore")
                state["tr"] = tr.value
                restored = b["t"].value
            ts = C.c_uint64(0)
            codec._check(lib.ckv_pipe_store_bf16_groups(
                pipe, src_ptrs, count, idx, sel, G, prefix, layers, epl, eps,
                slabs[k % 2].data_ptr(), cap, a["o"], a["s"], a["b"], C.byref(a["t"]),
                prev_restore, C.byref(ts), main.cuda_stream), "c3 store")
            state["ts"] = ts.value
            codec._check(lib.ckv_pipe_join(pipe, state["ts"], main.cuda_stream), "c3 join")
            main.wait_stream(side)
            return a["t"].value, restored

        for _ in range(3):
            step()
        times, totals = timed_steps(step, steps, flush, device)
        torch.cuda.synchronize(device)
        kms = [codec.kernel_ms(0), codec.kernel_ms(1)]

        # each direction alone: the store into slab 0, then its restore
        def store_only():
            main = torch.cuda.current_stream(device)
            a = meta[0]
            ts = C.c_uint64(0)
            codec._check(lib.ckv_pipe_store_bf16_groups(
                pipe, src_ptrs, count, idx, sel, G, prefix, layers, epl, eps,
                slabs[0].data_ptr(), cap, a["o"], a["s"], a["b"], C.byref(a["t"]),
                state["tr"], C.byref(ts), main.cuda_stream), "c3 store")
            state["ts"] = ts.value
            codec._check(lib.ckv_pipe_join(pipe, state["ts"], main.cuda_stream), "c3 join")

        def restore_only():
            main = torch.cuda.current_stream(device)
            b = meta[0]
            tr = C.c_uint64(0)
            codec._check(lib.ckv_pipe_restore_bf16_groups(
                pipe, slabs[0].data_ptr(), b["o"], b["s"], b["b"], count, idx, sel, G, prefix,
                layers, epl, dptr, state["ts"], C.byref(tr), main.cuda_stream), "c3 restore")
            state["tr"] = tr.value

        store_only()
        restore_only()
        dir_steps = min(steps, 3)
        t_st, _ = timed_steps(store_only, dir_steps, flush, device)
        t_rs, _ = timed_steps(restore_only, dir_steps, flush, device)
        torch.cuda.synchronize(device)
        t_d2h, t_h2d = raw_one_way(pages, dir_steps, flush, device)
        directions = direction_fields(1, raw_bytes, dir_steps, sum(t_st) / 1e3, sum(t_rs) / 1e3,
                                      raw_bytes, dir_steps, t_d2h, t_h2d)
        # the last restore read slab 0: check it against that store's
        # per-segment bounds
        last = meta[0]
        bnd = torch.tensor(list(last["b"]), device=device).view(count, G)
        owner = torch.zeros(layers, dtype=torch.long)
        owner[list(high)] = 1
        per_layer = bnd[:, owner.to(device)].view(count, 1, layers, 1)
        ok = True
        for c0 in range(0, count, 256):
            x = pages[c0:c0 + 256].float().view(-1, prefix, layers, epl)
            xh = dst[c0:c0 + 256].float().view(-1, prefix, layers, epl)
            ok &= bool(((x - xh).abs() <= per_layer[c0:c0 + 256] * 1.01 + 1e-7 +
                        x.abs() * 2.0 ** -8).all())
        stored = totals[-1][0]
        t = sum(times) / 1e3
        segment_ratio = [
            round(count * prefix * len(s) * epl * 2 / max(1, sum(list(meta[0]["s"])[g::G])), 4)
            for g, (_b, s) in enumerate(groups)]
        out = {
            "workload": f"C3: {count} pages x {codec.n} BF16 (the C2 pages x{repeat}), "
                        "7 layers at REL 1e-5 + 21 at REL 1e-4, two segments per page",
            "e2e_gbps": round(job_rate(1, raw_bytes, steps, t), 3),
            "overlapped_gbps": round(job_rate(1, raw_bytes, steps, t), 3),
            "ms_per_step": round(t * 1e3 / steps, 4),
            "compression_ratio": round(raw_bytes / stored, 4),
            "segment_ratios": {"1e-5": segment_ratio[0], "1e-4": segment_ratio[1]},
            "d2h_bytes_per_step": int(stored), "h2d_bytes_per_step": int(totals[-1][1]),
            "store_kernel_ms": round(kms[0], 4), "restore_kernel_ms": round(kms[1], 4),
            "restore_ok": ok,
            "path": "ckv_pipe_store_bf16_groups overlapped with ckv_pipe_restore_bf16_groups of "
                    f"the previous step's slab, {chunk_pages or count} pages per chunk",
        }
        out.update(directions)
        return out
    finally:
        torch.cuda.synchronize(device)
        lib.ckv_pipe_destroy(pipe)


# BASELINE.json configs[3] (C4: one job per request, 2048 pages) and configs[4] (C5, one GPU's
# 8192-page shard, moved as 16 jobs of 512 pages: the store of job k overlaps the restore of job
# k-1, so only the first store and the last restore run alone).
STREAMED = {
    "C4": {"layers": 28, "heads": 4, "jobs": 16, "pages_per_job": 2048, "eps": 1e-5, "seed": 1000,
           "what": "Qwen2.5-7B KV, 16 requests x 32k tokens (2048 pages each), REL 1e-5"},
    "C5": {"layers": 80, "heads": 1, "jobs": 16, "pages_per_job": 512, "eps": 1e-4, "seed": 2000,
           "what": "Llama-3-70B KV at 128k tokens, TP=8 shard of one GPU (8192 pages), REL 1e-4"},
}


def make_job_pages(layers: int, heads: int, pages: int, seed: int, device) -> torch.Tensor:
    """Seeded synthetic KV pages [pages, 2 * layers * heads * 16 * 128] BF16, generated on the
    device (the C2 distributions: K = N(0,1) x LogNormal(0, 0.5) per (layer, head, channel) with 4
    outlier channels x8, V = N(0, 0.5^2))."""
    g = torch.Generator(device=device).manual_seed(seed)
    kscale = torch.empty(layers, heads, HEAD_DIM, device=device).log_normal_(0.0, 0.5, generator=g)
    outliers = torch.randperm(HEAD_DIM, generator=g, device=device)[:4]
    kscale[:, :, outliers] *= 8.0
    out = torch.empty(pages, 2, layers, heads, TOKENS, HEAD_DIM, dtype=torch.bfloat16, device=device)
    for p0 in range(0, pages, 256):
        p1 = min(pages, p0 + 256)
        k = torch.randn(p1 - p0, layers, heads, TOKENS, HEAD_DIM, generator=g, device=device)
        out[p0:p1, 0] = (k * kscale[None, :, :, None, :]).to(torch.bfloat16)
        v = torch.randn(p1 - p0, layers, heads, TOKENS, HEAD_DIM, generator=g, device=device)
        out[p0:p1, 1] = (v * 0.5).to(torch.bfloat16)
    return out.view(pages, -1)


def streamed_shape(name: str, job_pages: int = 0) -> tuple:
    """(jobs, pages per job) of a C4 / C5 leg: the config's, or its pages split into jobs of
    job_pages pages."""
    cfg = STREAMED[name]
    if job_pages <= 0:
        return cfg["jobs"], cfg["pages_per_job"]
    total = cfg["jobs"] * cfg["pages_per_job"]
    if total % job_pages:
        raise ValueError(f"{name}: {total} pages do not split into jobs of {job_pages}")
    return total // job_pages, job_pages


def streamed_host_bytes(name: str, job_pages: int = 0) -> int:
    """Page-locked bytes a rank's C4 / C5 leg holds (two raw-size job slabs)."""
    cfg = STREAMED[name]
    pages_per_job = streamed_shape(name, job_pages)[1]
    return 2 * pages_per_job * 2 * cfg["layers"] * cfg["heads"] * TOKENS * HEAD_DIM * 2


def host_memory_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            return int(next(l for l in f if l.startswith("MemAvailable")).split()[1]) * 1024
    except (OSError, StopIteration, ValueError):
        return 0


def streamed_jobs(codec, name: str, steps: int, flush: torch.Tensor, device, rank: int = 0,
                  chunk_pages: int = 256, job_pages: int = 0, dist=None,
                  world: int = 1) -> dict:
    """C4 / C5 through the pipeline: a step stores every job (streamed_shape) from its own KV
    pages into one of two page-locked slabs on the caller's stream while the previous job is
    restored on a second stream (background store, on-demand restore), so the link carries a
    store and a restore at once.  Restores are checked per element against their page's bound.
    Each rank runs its own jobs (its own seeds, as a tensor-parallel shard would)."""
    cfg = STREAMED[name]
    lib, ck = codec.lib, codec.ckv
    jobs, pages_per_job = streamed_shape(name, job_pages)
    pages = [make_job_pages(cfg["layers"], cfg["heads"], pages_per_job,
                            cfg["seed"] + rank * jobs + r, device)
             for r in range(jobs)]
    n = pages[0].shape[1]
    dst = [torch.zeros_like(p) for p in pages]
    raw_job = pages_per_job * n * 2
    src_ptrs = [ck.ptr_array([p[i].data_ptr() for i in range(pages_per_job)]) for p in pages]
    dst_ptrs = [ck.ptr_array([d[i].data_ptr() for i in range(pages_per_job)]) for d in dst]
    eps = (C.c_float * pages_per_job)(*([cfg["eps"]] * pages_per_job))
    pipe = C.c_void_p()
    codec._check(lib.ckv_pipe_create(codec.ctx, chunk_pages, C.byref(pipe)), f"{name} pipe")
    try:
        # slabs of the raw job size: the synthetic pages compress by more than 1.3x (a job that
        # did not fit would fail the store with CKV_ERR_CAPACITY, not overrun)
        slabs = [torch.empty(raw_job, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        meta = [{"o": (C.c_size_t * pages_per_job)(), "s": (C.c_size_t * pages_per_job)(),
                 "b": (C.c_float * pages_per_job)(), "t": C.c_size_t(0)} for _ in range(jobs)]
        side = torch.cuda.Stream(device)
        last_reader = [0, 0]   # restore ticket that last read each slab
        stored = [0] * jobs

        def restore(r, after):
            side.wait_stream(torch.cuda.current_stream(device))
            t = C.c_uint64(0)
            m = meta[r]
            codec._check(lib.ckv_pipe_restore_bf16(
                pipe, slabs[r % 2].data_ptr(), m["o"], m["s"], m["b"], pages_per_job, n,
                dst_ptrs[r], after, C.byref(t), side.cuda_stream), f"{name} restore")
            last_reader[r % 2] = t.value

        def step():
            main = torch.cuda.current_stream(device)
            moved = 0
            for r in range(jobs + 1):
                if r >= 1:
                    restore(r - 1, stored[r - 1])
                if r < jobs:
                    t = C.c_uint64(0)
                    m = meta[r]
                    codec._check(lib.ckv_pipe_store_bf16(
                        pipe, src_ptrs[r], eps, pages_per_job, n, slabs[r % 2].data_ptr(), raw_job,
                        m["o"], m["s"], m["b"], C.byref(m["t"]), last_reader[r % 2], C.byref(t),
                        main.cuda_stream), f"{name} store")
                    stored[r] = t.value
                    moved += m["t"].value
            codec._check(lib.ckv_pipe_join(pipe, last_reader[(jobs - 1) % 2], main.cuda_stream),
                         f"{name} join")
            main.wait_stream(side)
            return moved

        step()
        if dist is not None:
            torch.cuda.synchronize(device)
            dist.barrier()
        times, moved = timed_steps(step, steps, flush, device)
        torch.cuda.synchronize(device)

        def check(r) -> bool:
            good = True
            b = torch.tensor(list(meta[r]["b"]), device=device).view(-1, 1)
            for p0 in range(0, pages_per_job, 256):
                x = pages[r][p0:p0 + 256].float()
                xh = dst[r][p0:p0 + 256].float()
                good &= bool(((x - xh).abs() <= b[p0:p0 + 256] * 1.01 + 1e-7 +
                              x.abs() * 2.0 ** -8).all())
            return good

        ok = all(check(r) for r in sorted({0, jobs - 1}))

        # each direction alone: every job stored (slab r % 2), then the last
        # two stored jobs restored alternately, `jobs` restores in all
        def store_only():
            main = torch.cuda.current_stream(device)
            for r in range(jobs):
                t = C.c_uint64(0)
                m = meta[r]
                codec._check(lib.ckv_pipe_store_bf16(
                    pipe, src_ptrs[r], eps, pages_per_job, n, slabs[r % 2].data_ptr(), raw_job,
                    m["o"], m["s"], m["b"], C.byref(m["t"]), last_reader[r % 2], C.byref(t),
                    main.cuda_stream), f"{name} store")
                stored[r] = t.value
            codec._check(lib.ckv_pipe_join(pipe, stored[jobs - 1], main.cuda_stream),
                         f"{name} join")

        def restore_only():
            main = torch.cuda.current_stream(device)
            for k in range(jobs):
                r = jobs - 2 + k % 2 if jobs > 1 else 0
                t = C.c_uint64(0)
                m = meta[r]
                codec._check(lib.ckv_pipe_restore_bf16(
                    pipe, slabs[r % 2].data_ptr(), m["o"], m["s"], m["b"], pages_per_job, n,
                    dst_ptrs[r], stored[r], C.byref(t), main.cuda_stream), f"{name} restore")
                last_reader[r % 2] = t.value

        def sync():
            torch.cuda.synchronize(device)
            if dist is not None:
                dist.barrier()

        store_only()
        sync()
        t_store, _ = timed_steps(store_only, 2, flush, device)
        restore_only()
        sync()
        t_rest, _ = timed_steps(restore_only, 2, flush, device)
        torch.cuda.synchronize(device)
        ok &= check(jobs - 1)
        sync()
        t_d2h, t_h2d = raw_one_way(pages[0], 2, flush, device, dist)
        t = sum(times) / 1e3
        raw_step = jobs * raw_job
        return {
            "workload": f"{name}: {cfg['what']}; {jobs} jobs x {pages_per_job} pages x {n} BF16 "
                        f"({raw_step / 1e9:.2f} GB), seeded on the device",
            "e2e_gbps": round(job_rate(1, raw_step, steps, t), 3),
            "ms_per_step": round(t * 1e3 / steps, 3),
            "seconds": t, "raw_bytes_per_step": raw_step, "steps": steps,
            "direction_seconds": [sum(t_store) / 1e3, sum(t_rest) / 1e3, t_d2h, t_h2d],
            "raw_sample_bytes": raw_job,
            "compression_ratio": round(raw_step / max(1, moved[-1]), 4),
            "d2h_bytes_per_step": int(moved[-1]), "h2d_bytes_per_step": int(moved[-1]),
            "restore_ok": ok,
            "path": "per job: ckv_pipe_store_bf16 on the caller's stream into one of two slabs, "
                    "overlapped with ckv_pipe_restore_bf16 of the previous job on a second stream; "
                    f"{chunk_pages} pages per chunk",
        }
    finally:
        torch.cuda.synchronize(device)
        lib.ckv_pipe_destroy(pipe)


def raw_pcie(pages_dev: torch.Tensor, steps: int, flush: torch.Tensor, device) -> float:
    """Raw pinned D2H + H2D of the uncompressed pages, one after the other (the
    PCIe reference point): seconds for `steps` steps of 2 x the pages' bytes."""
    pinned = torch.empty(pages_dev.numel() * 2, dtype=torch.uint8, pin_memory=True)
    src = pages_dev.view(-1).view(torch.uint8)
    back = torch.empty_like(src)

    def step():
        pinned.copy_(src, non_blocking=True)
        back.copy_(pinned, non_blocking=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize(device)
    times, _ = timed_steps(step, steps, flush, device)
    return sum(times) / 1e3


def raw_one_way(src: torch.Tensor, steps: int, flush: torch.Tensor, device,
                dist=None) -> tuple[float, float]:
    """Raw pinned copies of `src`'s bytes, one direction at a time: seconds
    for `steps` device-to-host copies, then for `steps` host-to-device
    copies (every rank at once under torchrun; the slowest rank's times)."""
    flat = src.reshape(-1).view(torch.uint8)
    pinned = torch.empty(flat.numel(), dtype=torch.uint8, pin_memory=True)
    back = torch.empty_like(flat)
    d2h = lambda: pinned.copy_(flat, non_blocking=True)   # noqa: E731
    h2d = lambda: back.copy_(pinned, non_blocking=True)   # noqa: E731
    for fn in (d2h, h2d):
        fn()
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    t_d2h, _ = timed_steps(d2h, steps, flush, device)
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    t_h2d, _ = timed_steps(h2d, steps, flush, device)
    del pinned, back
    return tuple(slowest_rank([sum(t_d2h) / 1e3, sum(t_h2d) / 1e3], dist, device))


def direction_fields(world: int, raw_bytes: int, steps: int, t_store: float, t_restore: float,
                     raw_sample: int, raw_steps: int, t_d2h: float, t_h2d: float) -> dict:
    """Store alone and restore alone (uncompressed bytes / device time, all
    ranks) next to raw one-way pinned copies of the same pages."""
    store = world * raw_bytes * steps / t_store / 1e9
    restore = world * raw_bytes * steps / t_restore / 1e9
    d2h = world * raw_sample * raw_steps / t_d2h / 1e9
    h2d = world * raw_sample * raw_steps / t_h2d / 1e9
    return {"store_gbps": round(store, 3), "restore_gbps": round(restore, 3),
            "raw_d2h_gbps": round(d2h, 3), "raw_h2d_gbps": round(h2d, 3),
            "store_vs_raw_d2h": round(store / d2h, 4), "restore_vs_raw_h2d": round(restore / h2d, 4)}


def slowest_rank(seconds: list[float], dist=None, device=None) -> list[float]:
    """Each timed region's duration on the slowest rank (max over ranks; the
    identity on one process)."""
    if dist is None:
        return list(seconds)
    t = torch.tensor(seconds, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def job_rate(world: int, raw_bytes: int, steps: int, seconds: float) -> float:
    """Whole-job GB/s: every rank stores and restores its raw_bytes each step."""
    return world * raw_bytes * 2 * steps / seconds / 1e9


def raw_pcie_duplex(pages_dev: torch.Tensor, steps: int, flush: torch.Tensor, device) -> float:
    """Raw pinned D2H and H2D of the uncompressed pages at the same time on two
    streams (the link ceiling for a store overlapped with a restore): seconds
    for `steps` steps of 2 x the pages' bytes."""
    src = pages_dev.view(-1).view(torch.uint8)
    pinned_out = torch.empty(src.numel(), dtype=torch.uint8, pin_memory=True)
    pinned_in = torch.empty(src.numel(), dtype=torch.uint8, pin_memory=True)
    back = torch.empty_like(src)
    s1 = torch.cuda.Stream(device)
    s2 = torch.cuda.Stream(device)
    main_stream = torch.cuda.current_stream(device)

    def step():
        s1.wait_stream(main_stream)
        s2.wait_stream(main_stream)
        with torch.cuda.stream(s1):
            pinned_out.copy_(src, non_blocking=True)
        with torch.cuda.stream(s2):
            back.copy_(pinned_in, non_blocking=True)
        main_stream.wait_stream(s1)
        main_stream.wait_stream(s2)

    for _ in range(2):
        step()
    torch.cuda.synchronize(device)
    times, _ = timed_steps(step, steps, flush, device)
    return sum(times) / 1e3


def bind_host_threads(physical: int, local: int, local_world: int):
    """Keeps this rank's host threads (and the page-locked memory they touch
    first) on CPUs of its own: the ones NVML names as closest to its GPU,
    and of the machine's CPUs the local rank's equal share, where the two
    overlap.  The timed steps wait on the host between the compress and the
    decompress calls, so a rank whose thread is preempted or shares a core
    with another rank's threads (torch keeps a pool of one thread per CPU in
    every process) stalls its GPU, and the slowest rank sets the number.
    Sets nothing on the GPU.  Returns the number of CPUs kept, or None."""
    try:
        import pynvml
        pynvml.nvmlInit()
        pynvml.nvmlDeviceSetCpuAffinity(pynvml.nvmlDeviceGetHandleByIndex(physical))
    except Exception:   # no NVML or no affinity information
        pass
    try:
        near = sorted(os.sched_getaffinity(0))
        cpus = list(range(os.cpu_count() or 1))
        per = max(1, len(cpus) // max(1, local_world))
        share = cpus[local * per:(local + 1) * per]
        mine = [c for c in share if c in near] or share
        os.sched_setaffinity(0, mine)
        torch.set_num_threads(len(mine))
        return len(mine)
    except Exception:
        return None


def host_info() -> dict:
    """The host's CPU count and model (/proc/cpuinfo), for the CPU baselines."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pages", type=int, default=PAGES)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c3", action="store_true",
                    help="skip the C3 mixed per-layer profile leg")
    ap.add_argument("--streamed", default="default",
                    help="comma-separated streamed legs: C4 (30 GB, 16 requests; one GPU), "
                         "C5 (5.4 GB TP=8 shard per GPU); 'default' runs C4 at N = 1 and C5 "
                         "at every N, 'none' neither")
    ap.add_argument("--chunk-pages", type=int, default=0,
                    help="pages per pipeline chunk (0: the whole job in one chunk)")
    ap.add_argument("--job-chunk-pages", type=int, default=256,
                    help="pages per pipeline chunk of the C4 / C5 jobs")
    ap.add_argument("--job-pages", type=int, default=0,
                    help="pages per job of the C4 / C5 legs (0: each config's own: C4 one "
                         "2048-page job per request, C5 16 jobs of 512 pages)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # on the host cores, rank 0 alone; the other ranks have nothing to do
        if rank == 0:
            print(json.dumps(reference_arm(args, world)))
        return 0
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v for v in visible.split(",") if v.strip()]
    physical = int(ids[local]) if len(ids) > local and ids[local].strip().isdigit() else local
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    affinity = bind_host_threads(physical, local, local_world) if world > 1 else None

    impl = args.impl

    host = make_pages(args.pages, seed=rank)
    raw_bytes = host.numel() * 2
    pages_dev = host.to(device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the CPU baseline: N = 1 only
        cpu = cpu_baseline(host)


    codec = (OurCodec(device, pages_dev, args.chunk_pages) if impl == "ours"
             else RefCodec(device, pages_dev))
    c3_slabs = (c3_host_slabs(codec) if impl == "ours" and rank == 0 and not args.no_c3
                else None)
    pipelined = impl == "ours"
    for _ in range(args.warmup):
        codec.step()
        codec.step_e2e()
        if pipelined:
            codec.step_e2e_pipelined()
    torch.cuda.synchronize(device)
    ok = codec.verify()

    def barrier():
        torch.cuda.synchronize(device)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    enc_ms, dec_ms, pack_ms = [], [], []

    def kernel_times():
        e = codec.kernel_ms(0)
        d = codec.kernel_ms(1)
        if e is not None:
            enc_ms.append(e)
            dec_ms.append(d)

    barrier()
    launches0 = codec.launches()
    # only rank 0's GPU is sampled (its line is the one printed): NVML queries
    # from every rank at 2 ms would contend with the ranks' own driver calls
    with ClockSampler(device, physical, enabled=rank == 0) as clocks:
        step_ms, _ = timed_steps(codec.step, args.steps, flush, device, after=kernel_times)
        barrier()
        launches_value = codec.launches() - launches0
        e2e_ms, totals = timed_steps(
            codec.step_e2e_pipelined if pipelined else codec.step_e2e, args.steps, flush, device)
        barrier()
        cont_s = None
        e2e_match = None
        if pipelined:
            e2e_match = codec.e2e_matches()
            cont_s, totals = codec.e2e_continuous(args.steps)
            e2e_match = e2e_match and codec.e2e_continuous_matches()
            barrier()
    launches_total = codec.launches() - launches0
    e2e_serial_ms = None
    c2_dirs = {}
    if pipelined:
        # the same step through the plain calls: compress, pack, one D2H, one
        # H2D, decompress, one after the other (outside the clock sampling)
        e2e_serial_ms, _ = timed_steps(codec.step_e2e, args.steps, flush, device)
        barrier()
        # each direction alone, next to raw one-way copies of the same pages
        for fn in (codec.step_store_only, codec.step_restore_only):
            fn()
        barrier()
        # each alone, steps back to back (inputs cycling through the three
        # copies of the pages), and each step synchronised with an L2 flush
        st_c = codec.run_continuous(
            lambda i: codec.step_store_only(pages_set=i % 3, join=False), args.steps)
        barrier()
        rs_c = codec.run_continuous(lambda i: codec.step_restore_only(), args.steps)
        barrier()
        st_ms, _ = timed_steps(codec.step_store_only, args.steps, flush, device)
        barrier()
        rs_ms, _ = timed_steps(codec.step_restore_only, args.steps, flush, device)
        barrier()
        t_d2h1, t_h2d1 = raw_one_way(pages_dev, min(args.steps, 10), flush, device, dist)
        t_st1, t_rs1, t_st_iso, t_rs_iso = slowest_rank(
            [st_c, rs_c, sum(st_ms) / 1e3, sum(rs_ms) / 1e3], dist, device)
        c2_dirs = direction_fields(world, raw_bytes, args.steps, t_st1, t_rs1, raw_bytes,
                                   min(args.steps, 10), t_d2h1, t_h2d1)
        c2_dirs["store_gbps_isolated"] = round(world * raw_bytes * args.steps / t_st_iso / 1e9, 3)
        c2_dirs["restore_gbps_isolated"] = round(world * raw_bytes * args.steps / t_rs_iso / 1e9, 3)
        barrier()
    if impl == "ours":
        pack_ms.append(codec.kernel_ms(2))
    compressed = codec.compressed_bytes()
    ok = ok and codec.verify()
    piped = (pipeline_codecs(codec, min(args.steps, 10), flush, device)
             if impl == "ours" and pipelined and rank == 0 else None)
    c1 = (c1_leg(codec, min(args.steps, 10), flush, device)
          if impl == "ours" and pipelined and rank == 0 else None)
    ref_kernels = (reference_kernels_leg(device, pages_dev, min(args.steps, 10), 3, flush,
                                         codec=codec)
                   if impl == "ours" and rank == 0 else None)
    c3 = None
    if impl == "ours" and pipelined and rank == 0 and not args.no_c3:
        # its page-locked slabs were prefaulted when allocated (a freshly
        # allocated 1 GiB slab pair used to run its first pass of copies at
        # half speed)
        c3 = layer_groups_c3(codec, min(args.steps, 10), flush, device,
                             chunk_pages=args.chunk_pages, slabs=c3_slabs)
    c1_pipe = (c1_pipeline(codec, min(args.steps, 10), flush, device)
               if impl == "ours" and pipelined and rank == 0 else None)
    plugin = (plugin_api_leg(codec, min(args.steps, 10), flush, device)
              if impl == "ours" and pipelined and rank == 0 else None)
    streamed = {}
    if args.streamed == "default":
        wanted = ["C4", "C5"] if world == 1 else ["C5"]
    elif args.streamed == "none":
        wanted = []
    else:
        wanted = [w.strip() for w in args.streamed.split(",") if w.strip()]
    for name in wanted:
        if impl != "ours" or not pipelined:
            continue
        # every rank runs its own shard; all ranks take the same branch
        fits = torch.tensor([1 if host_memory_available() >= world * 2 *
                             streamed_host_bytes(name, args.job_pages) else 0], device=device)
        if dist is not None:
            dist.all_reduce(fits, op=dist.ReduceOp.MIN)
        if not int(fits.item()):
            streamed[name] = {"workload": name, "skipped": "not enough host memory"}
            continue
        barrier()
        leg = streamed_jobs(codec, name, 3, flush, device, rank=rank, dist=dist, world=world,
                            job_pages=args.job_pages, chunk_pages=args.job_chunk_pages)
        t_st, t_rs, t_d2h, t_h2d = leg.pop("direction_seconds")
        (t_leg, t_st, t_rs) = slowest_rank([leg.pop("seconds"), t_st, t_rs], dist, device)
        leg["e2e_gbps_rank0"] = leg.pop("e2e_gbps")
        leg["e2e_gbps"] = round(job_rate(world, leg["raw_bytes_per_step"], leg["steps"], t_leg), 3)
        leg["overlapped_gbps"] = leg["e2e_gbps"]
        leg.update(direction_fields(world, leg["raw_bytes_per_step"], 2, t_st, t_rs,
                                    leg.pop("raw_sample_bytes"), 2, t_d2h, t_h2d))
        leg["n_gpus"] = world
        leg["gpus_active"] = world
        streamed[name] = leg
        gc.collect()
        torch.cuda.empty_cache()

    # every rank's device-resident step time (the line's value uses the slowest)
    step_by_rank = [statistics.median(step_ms)]
    if dist is not None:
        mine = torch.tensor([statistics.median(step_ms)], dtype=torch.float64, device=device)
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        step_by_rank = [float(x.item()) for x in allr]
    t_step, t_e2e_iso, t_serial, t_cont = slowest_rank(
        [sum(step_ms) / 1e3, sum(e2e_ms) / 1e3, sum(e2e_serial_ms) / 1e3 if e2e_serial_ms else 0.0,
         cont_s or 0.0], dist, device)
    t_e2e = t_cont if pipelined else t_e2e_iso
    value = job_rate(world, raw_bytes, args.steps, t_step)
    e2e = job_rate(world, raw_bytes, args.steps, t_e2e)
    e2e_iso = job_rate(world, raw_bytes, args.steps, t_e2e_iso)
    e2e_serial = job_rate(world, raw_bytes, args.steps, t_serial) if t_serial else None
    # the link ceilings at the same GPU count: every rank copies at once (GPUs
    # may share a PCIe switch and the host's memory), slowest rank's time
    raw_steps = min(args.steps, 10)
    barrier()
    t_raw = raw_pcie(pages_dev, raw_steps, flush, device)
    barrier()
    t_dup = raw_pcie_duplex(pages_dev, raw_steps, flush, device)
    barrier()
    t_raw, t_dup = slowest_rank([t_raw, t_dup], dist, device)
    pcie = world * 2 * pages_dev.numel() * 2 * raw_steps / t_raw / 1e9
    pcie_duplex = world * 2 * pages_dev.numel() * 2 * raw_steps / t_dup / 1e9

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return 0

    hbm, peak_kind = measured_hbm_gbs()
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step * 1e3 / args.steps, 4),
        "median_ms_per_step_by_rank": [round(x, 4) for x in step_by_rank],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32/u32",
        "data": "synthetic (seeded CPU generation, BASELINE.json configs[1] shapes)",
        "config": config_block(args.pages),
        "host_cpus_per_rank": affinity,
        "host": host_info(),
        "compression_ratio": round(raw_bytes / compressed, 4),
        "store_restore_ok": ok,
        "e2e": {"value": round(e2e, 3), "unit": "GB/s",
                "h2d_bytes_per_step": (int(totals[-1][1]) if pipelined else int(totals[-1]))
                if totals else compressed,
                "d2h_bytes_per_step": (int(totals[-1][0]) if pipelined else int(totals[-1]))
                if totals else compressed,
                "ms_per_step": round(t_e2e * 1e3 / args.steps, 4),
                "path": ("ckv_pipe_store_bf16 of step k's pages into one pinned slab, "
                         "overlapped with ckv_pipe_restore_bf16 of step k-1's slab; "
                         f"{codec.chunk} pages per chunk; the steps back to back with no "
                         "synchronisation between them, inputs cycling through three copies "
                         "of the pages (352 MB, more than L2) instead of an L2 flush") if pipelined else
                        "compress, torch.cat pack, one D2H, one H2D, decompress (in order)",
                "per_step_isolated_value": round(e2e_iso, 3) if pipelined else None,
                "per_step_isolated_ms": round(t_e2e_iso * 1e3 / args.steps, 4) if pipelined else None,
                "serial_value": round(e2e_serial, 3) if e2e_serial else None,
                "restore_matches_kernel_path": e2e_match,
                "pcie_raw_gbps": round(pcie, 3) if pcie else None,
                "pcie_raw_duplex_gbps": round(pcie_duplex, 3) if pcie_duplex else None,
                "fraction_of_raw_pcie": round(e2e / (pcie_duplex if pipelined else pcie), 4)
                if pcie and pcie_duplex else None,
                **c2_dirs},
    }
    if impl == "ours":
        enc = statistics.mean(enc_ms) / 1e3
        dec = statistics.mean(dec_ms) / 1e3
        enc_bytes = raw_bytes + compressed
        dec_bytes = compressed + raw_bytes
        kernels = {
            "encode": {"ms": round(enc * 1e3, 4), "gbps": round(enc_bytes / enc / 1e9, 2),
                       "frac": round(enc_bytes / enc / 1e9 / hbm, 4)},
            "decode": {"ms": round(dec * 1e3, 4), "gbps": round(dec_bytes / dec / 1e9, 2),
                       "frac": round(dec_bytes / dec / 1e9 / hbm, 4)},
        }
        if pack_ms:
            kernels["pack"] = {"ms": round(pack_ms[-1], 4)}
        dom, dom_t, dom_b = ("encode", enc, enc_bytes) if enc >= dec else ("decode", dec, dec_bytes)
        traffic, src = ncu_traffic(dom)
        line["roofline"] = {
            "bound": "hbm", "kernel": dom,
            "achieved": round(dom_b / dom_t / 1e9, 2), "peak": hbm, "unit": "GB/s",
            "frac": round(dom_b / dom_t / 1e9 / hbm, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6.65 TB/s",
            "traffic": traffic, "traffic_source": src,
            "algorithmic_bytes_per_launch": int(dom_b),
        }
        line["kernels"] = kernels
        line["pipeline_codecs"] = piped
        line["c1"] = c1
        line["c1_pipeline"] = c1_pipe
        line["plugin_api"] = plugin
        line["reference_kernels"] = ref_kernels
        line["layer_groups_c3"] = c3
        if streamed:
            line["streamed"] = streamed
        line["per_config"] = per_config_summary(world, line, c2_dirs, e2e, c1_pipe, c3, streamed)
        line["gpu_launches"] = launches_total
        line["gpu_launches_value_region"] = launches_value
    else:
        line["impl"] = "reference"
        line["reference_impl"] = ("the reference's batched BF16 kernels "
                                  "(integration/cuszp_wrapper/cuszp_batched_fixed.cu) "
                                  "built unchanged in oracle/_ref, driven like CuSZpWrapper")
        line["gpu_launches"] = None
    line["cpu_baseline"] = cpu
    if cpu is not None:
        line["codec_baselines"] = codec_baselines(host, pages_dev)
    line["clocks"] = clocks.summary()
    print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
