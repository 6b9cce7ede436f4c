"""Multi-rank host logic on CPU: world-size-2 gloo ranks (no GPU).

Checks that the per-rank shares of images and crops cover every item exactly
once and that the timing reduction returns the slowest rank's time, which is
what bench.py divides the whole job's units by.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ppocr_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        images = sharding.round_robin(37, world, rank)
        crops = list(sharding.even_split(4097, world, rank))
        gathered = [None] * world
        dist.all_gather_object(gathered, (images, crops))
        slowest = sharding.max_over_ranks(10.0 + rank)
        q.put((rank, gathered, slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_cover_the_work():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, slowest in results:
        assert slowest == 10.0 + (world - 1)
        images = sorted(i for g in gathered for i in g[0])
        crops = sorted(i for g in gathered for i in g[1])
        assert images == list(range(37))
        assert crops == list(range(4097))


def test_round_robin_and_even_split():
    assert sharding.round_robin(5, 2, 1) == [1, 3]
    assert list(sharding.even_split(10, 3, 0)) == [0, 1, 2, 3]
    assert list(sharding.even_split(10, 3, 2)) == [7, 8, 9]
    assert list(sharding.even_split(1, 4, 3)) == []
    with pytest.raises(ValueError):
        sharding.round_robin(3, 2, 2)


def test_width_buckets():
    widths = [160, 321, 100, 480, 320, 161]
    groups = sharding.width_buckets(widths, (480, 160, 320), batch=2)
    assert groups == [(160, [0, 2]), (320, [4, 5]), (480, [1, 3])]
    with pytest.raises(ValueError):
        sharding.width_buckets([481], (160, 320, 480), batch=4)


def test_max_over_ranks_without_group():
    assert sharding.max_over_ranks(3.5) == 3.5
