"""Multi-rank host logic on CPU: page sharding, disjoint global page ranges and the max-over-ranks timing
reduction, run as two gloo ranks (127.0.0.1)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from ztcp_b200 import sharding


def test_shard_range_covers_exactly():
    for n in (0, 1, 7, 256, 4096, 4097):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            assert sum(c for _, c in spans) == n
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def test_global_page_base_disjoint():
    seen = set()
    for rank in range(8):
        for batch in range(4):
            b = sharding.global_page_base(rank, batch, 4, 256)
            pages = set(range(b, b + 256))
            assert not (pages & seen)
            seen |= pages
    assert seen == set(range(8 * 4 * 256))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = sharding.shard_range(4096, world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, (start, count))
        ms = sharding.max_over_ranks([1.0 + rank, 10.0 - rank])
        out[rank] = (gathered, ms)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        res = dict(out)
    for rank in range(world):
        gathered, ms = res[rank]
        assert gathered == [(0, 2048), (2048, 2048)]
        assert ms == [2.0, 10.0]
