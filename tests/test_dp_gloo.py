"""Host logic of the multi-GPU path on CPU: world_size-2 gloo process group.
Every image is encoded by exactly one rank (the shards tile the batch), the
shards are balanced, seeds agree across ranks, and the step time reported is
the max over ranks."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import dp


def test_shard_range_tiles_the_batch():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            got = [dp.shard_range(n, world, r) for r in range(world)]
            covered = [i for first, cnt in got for i in range(first, first + cnt)]
            assert covered == list(range(n))
            cnts = [c for _, c in got]
            assert max(cnts) - min(cnts) <= 1
    with pytest.raises(ValueError):
        dp.shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first, cnt = dp.shard_range(64, world, rank)
    mine = torch.zeros(64, dtype=torch.int64)
    mine[first:first + cnt] = 1
    dist.all_reduce(mine)  # every image claimed exactly once
    seeds = torch.tensor([dp.image_seed(i) for i in range(first, first + cnt)])
    t = dp.max_over_ranks(10.0 * (rank + 1))
    q.put((rank, mine.tolist(), seeds.tolist(), t))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mine, seeds, t in res:
        assert mine == [1] * 64
        assert t == 20.0
    assert res[0][2] == list(range(100, 132)) and res[1][2] == list(range(132, 164))
