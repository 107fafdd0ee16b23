"""bench.py's multi-rank plumbing on CPU with the gloo backend (world size 2): every rank
takes the same collective steps and rank 0 reports the maximum over ranks."""
import os
import socket
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import bench
    dist = bench.Dist("gloo")
    dist.barrier()
    value = dist.max(1.5 + rank)          # per-rank timing; the job's time is the slowest rank
    total = dist.max(float(rank * 10))
    frames = dist.sum(float(64 * (rank + 1)))   # every rank's frames count toward the job's value
    dist.barrier()
    dist.close()
    out.put((rank, value, total, frames))


def test_gloo_world_size_two_takes_max_over_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == [(0, 2.5, 10.0, 192.0), (1, 2.5, 10.0, 192.0)]
