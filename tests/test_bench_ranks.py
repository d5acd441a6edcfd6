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
