"""The multi-GPU host logic (wocr/shard.py) on CPU: page partition, and the barrier and
max-over-ranks reduction with two gloo ranks (the GPU run uses the same calls over nccl)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from wocr.shard import max_over_ranks, pages_of, weak_pages_of


@pytest.mark.parametrize("n,world", [(12, 1), (12, 2), (12, 8), (96, 8), (7, 3), (2, 4)])
def test_pages_partition(n, world):
    parts = [pages_of(r, world, n) for r in range(world)]
    flat = [p for part in parts for p in part]
    assert flat == list(range(n))                       # disjoint, complete, in order
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1                  # balanced


def test_weak_pages():
    assert weak_pages_of(0, 12) == list(range(12))
    assert weak_pages_of(3, 12) == list(range(36, 48))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    from wocr.shard import barrier
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = pages_of(rank, world, 12)
        barrier()
        t = max_over_ranks(1.0 + rank * 2.5)            # stand-in device times
        got = [None] * world
        dist.all_gather_object(got, mine)
        out.put((rank, t, got))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, t, got in res:
        assert t == 1.0 + (world - 1) * 2.5               # the max over ranks on every rank
        assert [x for part in got for x in part] == list(range(12))
