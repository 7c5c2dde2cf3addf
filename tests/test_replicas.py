"""Multi-process (gloo, world size 2) check of the bench's replica aggregation:
one process per GPU in production, CPU ranks here."""
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
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    maxed, summed = bench.reduce_over_ranks([10.0 + rank, 1.5 * (rank + 1)], [240, 1000 + rank],
                                            world, "cpu")
    out[rank] = (maxed, summed)
    dist.destroy_process_group()


def test_reduce_over_ranks_gloo():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        maxed, summed = res[r]
        assert maxed == [11.0, 3.0]  # slowest replica's times
        assert summed == [480.0, 2001.0]  # frames and launches over all replicas


def test_reduce_over_ranks_single():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.reduce_over_ranks([1.0, 2.0], [3, 4], 1, "cpu") == ([1.0, 2.0], [3, 4])
