"""CPU tests of the data-parallel host logic with world_size-2 gloo ranks:
sharding covers every sequence exactly once, and the max-over-ranks timing
reduction sees every rank."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from c_gpt2_b200.dp import shard


def test_shard_covers_all():
    for n in (1, 7, 64, 65):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                first, count = shard(n, r, world)
                seen += list(range(first, first + count))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from c_gpt2_b200.dp import max_over_ranks, shard, sum_over_ranks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _, count = shard(64, rank, world)
        total = sum_over_ranks(count)
        slowest = max_over_ranks(10.0 + rank)
        dist.barrier()
        q.put((rank, total, slowest))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_max_and_sum():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res == [(0, 64.0, 11.0), (1, 64.0, 11.0)]
