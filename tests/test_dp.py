"""Data-parallel host logic (no GPU): the sequence partitioner and the job-level
reductions, the latter across two gloo processes on 127.0.0.1."""
import os
import socket

import numpy as np
import pytest

from yanaiengine_b200 import dp


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partition_covers_each_sequence_once(world):
    lengths = dp.global_lengths(32, world, seed=5)
    parts = dp.partition(lengths, world)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(lengths)))
    cap = -(-len(lengths) // world)
    assert all(len(p) <= cap for p in parts)
    loads = [int(lengths[p].sum()) for p in parts]
    # count-capped longest-first stays within the greedy bound of the mean
    assert max(loads) <= 4 / 3 * np.mean(loads) + lengths.max()


def test_partition_is_deterministic_and_balanced():
    lengths = np.array([2048, 2040, 512, 520, 1000, 1100, 1500, 900])
    a, b = dp.partition(lengths, 2), dp.partition(lengths, 2)
    assert a == b
    loads = [int(lengths[p].sum()) for p in a]
    assert abs(loads[0] - loads[1]) <= 600
    assert [len(p) for p in a] == [4, 4]


def test_partition_edge_cases():
    assert dp.partition([], 2) == [[], []]
    assert dp.partition([7], 4) == [[0], [], [], []]
    with pytest.raises(ValueError):
        dp.partition([1, 2], 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lengths = dp.global_lengths(32, world, seed=9)
        mine = dp.partition(lengths, world)[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        slowest = dp.all_max(world, 10.0 + rank, device="cpu")
        total = dp.all_sum(world, float(len(mine)), device="cpu")
        q.put((rank, gathered, slowest, total))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_partition_and_reductions():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, slowest, total in results:
        flat = sorted(i for part in gathered for i in part)
        assert flat == list(range(64))  # every sequence on exactly one rank
        assert slowest == 11.0          # max over ranks of the device time
        assert total == 64.0            # sum of per-rank counts
