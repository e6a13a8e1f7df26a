"""Multi-process host logic of the clip-sharded (weak-scaling) benchmark on
CPU: two gloo ranks, no GPU. Every rank gets its own contiguous clips, the
shards cover the batch exactly once, and the job time is the slowest rank's.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp

from wxb200 import dist as D


def test_shard_covers_every_clip_once():
    for n in (0, 1, 7, 64, 65):
        for w in (1, 2, 3, 8):
            spans = [D.shard(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        D.shard(4, 2, 2)


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
        D.barrier()
        w, r = D.world()
        t = D.max_over_ranks(1.0 + rank)          # rank 1 is the slow one
        clips = D.sum_over_ranks(D.shard(64, w, r)[1] - D.shard(64, w, r)[0])
        per_rank = D.gather_to_all({"rank": rank, "ms": 10.0 * (rank + 1)})
        q.put((rank, w, r, t, clips, per_rank))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_barrier_max_and_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out = sorted(q.get(timeout=10) for _ in range(2))
    for rank, w, r, t, clips, per_rank in out:
        assert (w, r) == (2, rank)
        assert t == 2.0          # max over ranks
        assert clips == 64       # the shards add up to the batch
        assert per_rank == [{"rank": 0, "ms": 10.0}, {"rank": 1, "ms": 20.0}]
