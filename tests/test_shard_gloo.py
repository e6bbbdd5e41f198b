"""Multi-process host logic of the sharded batch path on CPU: two gloo ranks (127.0.0.1).

Checks that the shard ranges of all ranks tile the batch exactly once and that the timing reductions used
by bench.py (max over ranks of the step time, sum of per-rank payload) agree on every rank.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp

from dsmem_b200.shard import max_over_ranks, shard_range, sum_over_ranks


def test_shard_range_tiles_the_batch():
    for total in (0, 1, 7, 8, 4096, 4099):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                s, c = shard_range(total, r, world)
                covered.extend(range(s, s + c))
            assert covered == list(range(total))
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = shard_range(1000, rank, world)
        t = max_over_ranks(1.5 + rank, dist)
        total = sum_over_ranks(count, dist)
        q.put((rank, start, count, t, total))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert [r[1] for r in res] == [0, 500] and [r[2] for r in res] == [500, 500]
    assert all(r[3] == 2.5 for r in res)          # max over ranks
    assert all(r[4] == 1000 for r in res)         # payload summed over ranks
