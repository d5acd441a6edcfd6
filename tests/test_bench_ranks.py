"""bench.py's multi-process host logic on CPU (gloo, two ranks).

With N GPUs each rank times its own shard; the reported value is the total
over ranks divided by the SLOWEST rank's time.  Two gloo processes stand in
for two GPUs: they report different durations and must both see the
maximum, and the job rate must count both ranks' bytes.
"""
import os
import socket
import sys
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = [1.0 + rank, 3.0 - rank, 0.5 * (rank + 1)]
        out[rank] = bench.slowest_rank(mine, dist, torch.device("cpu"))
    finally:
        dist.destroy_process_group()


def test_two_ranks_report_the_slowest():
    world = 2
    port = _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        got = dict(out)
    assert got[0] == got[1] == [2.0, 3.0, 1.0]


def test_job_rate_counts_every_rank():
    sys.path.insert(0, str(ROOT))
    import bench

    one = bench.job_rate(1, 117440512, 10, 0.01)
    assert abs(bench.job_rate(4, 117440512, 10, 0.01) - 4 * one) < 1e-9
    assert abs(one - 2 * 117440512 * 10 / 0.01 / 1e9) < 1e-9
    assert bench.slowest_rank([1.0, 2.0]) == [1.0, 2.0]


def test_reference_arm_line_on_cpu():
    """The reference arm runs on the host cores alone and prints the contract's
    keys: impl, a cpu_baseline describing the run with value = the line's,
    and an e2e with no copies."""
    import argparse
    sys.path.insert(0, str(ROOT))
    import bench

    args = argparse.Namespace(pages=2, steps=1, warmup=1)
    line = bench.reference_arm(args, world=2)
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] == "port" and cb["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert 1.0 < line["compression_ratio"] < 3.0
