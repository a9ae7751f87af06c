"""World-size-2 gloo test of the multi-GPU host logic (session sharding and
max-over-ranks timing) on CPU processes."""
import os
import socket

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from funasrnet_b200.shard import assign_sessions, max_over_ranks, sum_over_ranks, throughput

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    mine = assign_sessions(2048, world, rank)
    n = sum_over_ranks(len(mine), dist)
    slowest = max_over_ranks(1.0 + rank, dist)
    dist.barrier()
    q.put((rank, mine[:3], n, slowest, throughput(128, world, slowest)))
    dist.destroy_process_group()


def test_two_rank_sharding_and_timing():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, s0, n0, m0, t0), (r1, s1, n1, m1, t1) = results
    assert s0 == [0, 2, 4] and s1 == [1, 3, 5]
    assert n0 == n1 == 2048
    assert m0 == m1 == 2.0          # the slowest rank sets the time
    assert t0 == t1 == 128 * 2 / 2.0


def test_assign_sessions_partition():
    from funasrnet_b200.shard import assign_sessions

    for world in (1, 2, 4, 8):
        owned = sorted(i for r in range(world) for i in assign_sessions(2048, world, r))
        assert owned == list(range(2048))
    with pytest.raises(ValueError):
        assign_sessions(10, 2, 2)
