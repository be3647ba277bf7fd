"""Multi-GPU replicas, host logic on CPU: world_size-2 gloo ranks.

bench.py runs one independent pager per GPU (no data-path collective); the
process group carries only the timing barrier and the max/sum reductions of the
per-rank figures.  These ranks use gloo on CPU with made-up per-rank figures.
"""

import os
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.barrier(world)
        moved = 1e9 * (rank + 1)  # rank r moved (r+1) GB
        ms = 100.0 + 50.0 * rank  # the slowest rank takes 150 ms
        out[rank] = bench.aggregate(moved, ms, world)
    finally:
        dist.destroy_process_group()


def test_replica_aggregation_over_gloo():
    world = 2
    port = 29600 + os.getpid() % 200
    with mp.get_context("spawn").Manager() as m:  # no fork of a threaded process
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        gbs, total, ms_max = res[r]
        assert total == pytest.approx(3e9) and ms_max == pytest.approx(150.0)
        assert gbs == pytest.approx(3e9 / 0.150 / 1e9)
