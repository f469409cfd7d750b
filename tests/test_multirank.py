"""The multi-GPU path's host logic, on two gloo ranks on the CPU.

A single image does not shard (grid gating mixes the whole image), so the
scale-out is replicas: image i of the seeded stream goes to rank i % N, each
rank runs its own executor, and the only collective is the max over ranks of
the timed region. These run that logic (bench.py's own helpers) as two real
processes over torch.distributed with the gloo backend.
"""
import importlib
import os
import socket
import sys
from datetime import timedelta

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        sys.path.insert(0, ROOT)
        bench = importlib.import_module("bench")
        mine = bench.shard(3, rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, mine)
        slowest = bench.max_over_ranks(1.0 + rank, world)  # the last rank is the slow one
        value = bench.job_mpx_per_s(3, world, slowest)
        # The reference arm: every rank but 0 leaves without work or output.
        quiet = rank == 0 or bench.run_reference(None) == 0
        dist.barrier()
        q.put((rank, shards, slowest, value, quiet, bench.OUT_MPX))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_replicas_shard_images_and_take_the_slowest_rank():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_rank_main, args=(world, _free_port(), q), nprocs=world, join=True)
    got = sorted(q.get(timeout=30) for _ in range(world))
    for rank, shards, slowest, value, quiet, out_mpx in got:
        # Disjoint shards that cover the stream, image i on rank i % N.
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(3 * world))
        assert all(i % world == r for r, s in enumerate(shards) for i in s)
        # Every rank sees the slowest rank's time, and the job's throughput
        # counts every rank's images over it.
        assert slowest == float(world)
        assert value == pytest.approx(3 * world * out_mpx / world)
        assert quiet
