"""Host-side multi-GPU logic on the CPU: LPT event sharding and the rank-order
collectives, run as world_size-2 gloo process groups."""

import os
import random

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_spacetime.sharding import (
    gather_over_ranks,
    gather_rows,
    lpt_partition,
    max_over_ranks,
    ordered_sum,
    pack_events,
    shard_loads,
)
from flash_spacetime.synthetic import lengths_for


def test_lpt_partition_covers_and_balances():
    lens = lengths_for("config3", 4096, seed=3)
    for world in (1, 2, 4, 8):
        shards = lpt_partition(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))
        loads = shard_loads(lens, shards)
        # Longest-first greedy: max load within one largest event of the mean.
        mean = sum(loads) / world
        assert max(loads) - mean <= max(int(n) ** 2 for n in lens)
        assert max(loads) / mean < 1.05


def test_lpt_partition_is_deterministic():
    lens = [random.Random(1).randint(1, 3000) for _ in range(1000)]
    assert lpt_partition(lens, 4) == lpt_partition(list(lens), 4)


def test_pack_events():
    lens, cu = pack_events([5, 1, 7, 3], [2, 0])
    assert lens == [7, 5]
    assert cu.tolist() == [0, 7, 12]
    assert cu.dtype == torch.int32


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = torch.arange(6, dtype=torch.float32) * (rank + 1)
        s = ordered_sum(t)
        rows = gather_rows(torch.full((rank + 2, 3), float(rank)))
        # Host-known sizes (every rank computes the same partition): no size exchange.
        rows2 = gather_rows(torch.full((rank + 2, 3), float(rank)), sizes=[2, 3])
        assert [r.tolist() for r in rows2] == [r.tolist() for r in rows]
        m = max_over_ranks(float(rank) * 1.5, torch.device("cpu"))
        assert gather_over_ranks(float(rank) * 1.5, torch.device("cpu")) == [0.0, 1.5]
        q.put((rank, s.tolist(), [r.tolist() for r in rows], m))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random(os.getpid()).randint(0, 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, s, rows, m = q.get(timeout=120)
        got[rank] = (s, rows, m)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect_sum = [float(3 * i) for i in range(6)]
    for rank in (0, 1):
        s, rows, m = got[rank]
        assert s == expect_sum
        assert [len(r) for r in rows] == [2, 3]
        assert rows[1][0] == [1.0, 1.0, 1.0]
        assert m == 1.5
    assert got[0] == got[1]
