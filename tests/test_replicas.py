"""The replica partition and the job timing across ranks: two gloo processes on the CPU."""
import os

import pytest

from hwnpu_b200 import replicas

torch = pytest.importorskip("torch")


def test_shard_partitions_round_robin():
    for n in (0, 1, 7, 64):
        for world in (1, 2, 3, 8):
            parts = [replicas.shard(n, r, world) for r in range(world)]
            assert sorted(i for p in parts for i in p) == list(range(n))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = replicas.shard(64, rank, world)
        # a replica's time and token count: the job sees the slowest and the total
        t = replicas.job_time(1.0 + rank, dist)
        n = replicas.job_total(len(mine), dist)
        q.put((rank, mine, t, n))
    finally:
        dist.destroy_process_group()


def test_two_ranks_gloo():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, m0, t0, n0), (r1, m1, t1, n1) = res
    assert m0 == list(range(0, 64, 2)) and m1 == list(range(1, 64, 2))
    assert t0 == t1 == 2.0
    assert n0 == n1 == 64
