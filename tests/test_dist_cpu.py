"""Multi-process (gloo, world size 2, CPU) checks of the sharding and timing reductions used at N > 1."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from wgkv.dist import kv_head_shard, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 16, 64, 1000):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    assert kv_head_shard(8, 32, 3, 8) == ((3, 4), (12, 16))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from wgkv.dist import max_over_ranks, shard_range, sum_over_ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, end = shard_range(16 * world, rank, world)
        mx = max_over_ranks(10.0 + rank)
        total = sum_over_ranks(end - start)
        q.put((rank, start, end, mx, total))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_reductions():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(r[1], r[2]) for r in res] == [(0, 16), (16, 32)]
    assert all(r[3] == 11.0 for r in res)  # max over ranks of 10 + rank
    assert all(r[4] == 32 for r in res)
