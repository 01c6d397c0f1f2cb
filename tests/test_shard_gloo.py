"""Multi-rank host logic on CPU (gloo, world size 2): sequence sharding and timing."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rwkv_tl_b200.shard import gather_to_rank0, max_over_ranks, shard_by_length, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 256, 2048):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert sum(len(p) for p in parts) == n
            assert [i for p in parts for i in p] == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_shard_by_length_balances_tokens():
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(16, 2049, (2048,), generator=g).tolist()  # config 4 prompt lengths
    parts = shard_by_length(lens, 8)
    assert sorted(i for p in parts for i in p) == list(range(2048))
    loads = [sum(lens[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(lens)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = list(shard_range(10, world, rank))
        t = max_over_ranks(1.0 + rank)
        got = gather_to_rank0(mine)
        if rank == 0:
            q.put((t, got))
    finally:
        dist.destroy_process_group()


def test_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    t, got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert t == 2.0
    assert got == [[0, 1, 2, 3, 4], [5, 6, 7, 8, 9]]


def test_single_process_fallbacks():
    assert max_over_ranks(3.5) == 3.5
    assert gather_to_rank0({"a": 1}) == [{"a": 1}]
