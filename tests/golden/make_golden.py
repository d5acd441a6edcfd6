"""Generate the golden fixtures from the reference's own kernels (GPU).

Runs the reference's batched fixed-mode BF16 kernels (built from its
integration/cuszp_wrapper/cuszp_batched_fixed.cu into oracle/_ref by
oracle/build.py) on every case in cases.py and stores, per case:

* the compressed bytes of every unit (the kernels' own output, with the
  compressed buffers zeroed before the call so the rate bytes the
  reference never writes are zero), their sizes and resolved bounds;
* the decoded BF16 of every unit, decoded by the reference's own decoder
  from its own bitstream into destinations prefilled with SENTINEL (blocks
  whose rate is zero are not written by the reference decoder, so they keep
  the sentinel): per-page scatter mode for plain cases (destination
  split in destinations_per_page parts), layer-indexed scatter for indexed
  cases, and the contiguous [batch][n] mode where n is even;
* which form of the quantiser (separate or fused multiply-add) the C
  oracle needs to reproduce the bytes.

Usage (on a GPU box):  python tests/golden/make_golden.py OUT_DIR
The files in OUT_DIR are then copied into tests/golden/fixtures/.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from cases import CASES, Case, inputs_sha256, unit_bits  # noqa: E402
from oracle.oracle import COracle, RefKernels, capacity_for, header_bytes  # noqa: E402

SENTINEL = 0x3F81  # BF16 1.0078125


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def run_case(ref: RefKernels, co: COracle, case: Case, dev: torch.device):
    n = case.n
    src_numel = case.source_numel
    pages = [torch.from_numpy(unit_bits(case, u).view(np.int16)).to(dev)
             .view(torch.bfloat16) for u in range(case.batch)]
    cap = max(8 * n, capacity_for(n))
    outs = [torch.empty(cap, dtype=torch.uint8, device=dev) for _ in pages]
    eps = [case.eps_of(u) for u in range(case.batch)]
    layer_ptr = None
    idx_t = None
    if case.layer_indices is not None:
        idx_t = torch.tensor(case.layer_indices, dtype=torch.int64, device=dev)
        layer_ptr = idx_t.data_ptr()
    sizes, bounds = ref.compress(
        [p.data_ptr() for p in pages], [o.data_ptr() for o in outs], cap, n, eps,
        relative=case.relative, layer_indices_ptr=layer_ptr,
        selected=len(case.layer_indices or ()), prefix_count=case.prefix_count,
        source_layers=case.source_layers,
        elements_per_layer=case.elements_per_layer)
    torch.cuda.synchronize()
    comp = [outs[u][: int(sizes[u])].cpu().numpy() for u in range(case.batch)]

    result = {
        "sizes": sizes.astype(np.int64),
        "bounds": bounds.astype(np.float32),
        "compressed": np.concatenate(comp),
    }

    # Decode with the reference decoder from its own bitstream.
    in_ptrs = [o.data_ptr() for o in outs]
    if case.layer_indices is not None:
        dests = [torch.full((src_numel,), SENTINEL, dtype=torch.int16, device=dev)
                 .view(torch.bfloat16) for _ in pages]
        ref.decompress(in_ptrs, n, bounds, 2, [d.data_ptr() for d in dests],
                       layer_indices_ptr=layer_ptr,
                       selected=len(case.layer_indices),
                       prefix_count=case.prefix_count,
                       source_layers=case.source_layers,
                       elements_per_layer=case.elements_per_layer)
        torch.cuda.synchronize()
        result["decoded"] = np.stack(
            [d.view(torch.int16).cpu().numpy().view(np.uint16) for d in dests])
    else:
        per = case.destinations_per_page
        epd = n // per
        assert epd * per == n
        dests = [torch.full((epd,), SENTINEL, dtype=torch.int16, device=dev)
                 .view(torch.bfloat16) for _ in range(case.batch * per)]
        ref.decompress(in_ptrs, n, bounds, 1, [d.data_ptr() for d in dests],
                       per_page=per, elements_per_dest=epd)
        torch.cuda.synchronize()
        flat = np.concatenate(
            [d.view(torch.int16).cpu().numpy().view(np.uint16) for d in dests])
        result["decoded"] = flat.reshape(case.batch, n)
        if n % 2 == 0:
            # The contiguous launcher stores BF16 pairs at page * n + i, which
            # is only 4-byte aligned for even n.
            out = torch.full((case.batch * n,), SENTINEL, dtype=torch.int16,
                             device=dev).view(torch.bfloat16)
            ref.decompress(in_ptrs, n, bounds, 0, [out.data_ptr()])
            torch.cuda.synchronize()
            cont = out.view(torch.int16).cpu().numpy().view(np.uint16)
            result["decoded_contiguous"] = cont.reshape(case.batch, n)

    # Which quantiser form reproduces the reference bytes?
    match = {}
    for fused in (False, True):
        ok = True
        for u in range(case.batch):
            bits = unit_bits(case, u)
            kw = {}
            if case.layer_indices is not None:
                kw = dict(layer_indices=case.layer_indices,
                          prefix_count=case.prefix_count,
                          source_layers=case.source_layers,
                          elements_per_layer=case.elements_per_layer)
            buf, eb = co.encode(bits, eps[u], relative=case.relative,
                                fused=fused, **kw)
            if (buf.size != comp[u].size or not np.array_equal(buf, comp[u])
                    or np.float32(eb).tobytes() != bounds[u].tobytes()):
                ok = False
        match["fused" if fused else "separate"] = ok
    return result, match


def main(out_dir: str) -> int:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    ref = RefKernels()
    co = COracle()
    manifest = {"sentinel": SENTINEL, "cases": {}}
    for case in CASES:
        result, match = run_case(ref, co, case, dev)
        np.savez_compressed(out / f"{case.name}.npz", **result)
        entry = {
            "inputs_sha256": inputs_sha256(case),
            "sizes": [int(s) for s in result["sizes"]],
            "bounds_hex": [np.float32(b).tobytes().hex() for b in result["bounds"]],
            "compressed_sha256": _sha(result["compressed"]),
            "decoded_sha256": _sha(result["decoded"]),
            "oracle_match": match,
            "header_bytes": header_bytes(case.n),
        }
        if "decoded_contiguous" in result:
            entry["contiguous_equals_scatter"] = bool(np.array_equal(
                result["decoded_contiguous"], result["decoded"]))
        manifest["cases"][case.name] = entry
        print(case.name, entry["sizes"], match, flush=True)
    manifest["device"] = torch.cuda.get_device_name(0)
    manifest["torch"] = torch.__version__
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else "golden_out"))
