"""Batch x head partitioning arithmetic (host side, no GPU), on one process and on two gloo ranks."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sbda_b200.partition import rank_views, unit_pieces, unit_range


@pytest.mark.parametrize("batch,kv_heads", [(8, 8), (3, 4), (1, 5), (5, 1), (0, 4), (7, 3)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_ranges_cover_every_unit_once(batch, kv_heads, world):
    seen = []
    sizes = []
    for rank in range(world):
        lo, hi = unit_range(batch, kv_heads, world, rank)
        sizes.append(hi - lo)
        units = []
        for b0, b1, h0, h1 in unit_pieces(lo, hi, kv_heads):
            assert 0 <= b0 < b1 <= batch and 0 <= h0 < h1 <= kv_heads
            assert b1 - b0 == 1 or (h0, h1) == (0, kv_heads)
            units += [b * kv_heads + h for b in range(b0, b1) for h in range(h0, h1)]
        assert units == list(range(lo, hi))
        seen += units
    assert seen == list(range(batch * kv_heads))
    assert max(sizes) - min(sizes) <= 1


def test_views_alias_the_callers_tensors():
    q = torch.zeros(3, 8, 10, 4)          # H = 8, Hkv = 4 (G = 2)
    k = torch.zeros(3, 4, 10, 4)
    lse = torch.zeros(3, 8, 10)
    for rank in range(5):
        for (qv, lv), (kv,) in rank_views((q, lse), (k,), 5, rank):
            qv.add_(1)
            lv.add_(1)
            kv.add_(1)
            assert qv.data_ptr() >= q.data_ptr() and lv.is_contiguous()
            assert qv.shape[1] == 2 * kv.shape[1]
    assert torch.equal(q, torch.ones_like(q)) and torch.equal(k, torch.ones_like(k))
    assert torch.equal(lse, torch.ones_like(lse))


def test_bad_arguments():
    with pytest.raises(ValueError):
        unit_range(4, 4, 0, 0)
    with pytest.raises(ValueError):
        unit_range(4, 4, 2, 2)
    with pytest.raises(ValueError):
        rank_views((torch.zeros(1, 3, 4, 2),), (torch.zeros(1, 2, 4, 2),), 1, 0)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        batch, kv_heads = 3, 5
        mine = unit_range(batch, kv_heads, world, rank)
        ranges = [None] * world
        dist.all_gather_object(ranges, mine)
        # ranges tile [0, B * Hkv) in rank order, and each rank's views touch only its units
        assert ranges[0][0] == 0 and ranges[-1][1] == batch * kv_heads
        assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
        mark = torch.zeros(batch, kv_heads, 1, 1)
        for _, (kv,) in rank_views((torch.zeros(batch, kv_heads, 1, 1),), (mark,), world, rank):
            kv.fill_(rank + 1)
        dist.all_reduce(mark)
        expected = torch.tensor([r + 1 for r in range(world) for _ in range(*ranges[r])], dtype=mark.dtype)
        assert torch.equal(mark.flatten(), expected)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_the_units():
    mp.spawn(_worker, args=(2, _port()), nprocs=2, join=True)
