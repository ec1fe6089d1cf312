"""Host-side shard arithmetic on two gloo ranks (no GPU): shards partition the sequence and
every rank agrees on the owner of every position, including the dyadic sources and consumers
the sharded kernels fetch from other ranks."""

from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sbda_b200.sharded import owner_of, shard_bounds

TOTAL = 4096


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = shard_bounds(TOTAL, world, rank)
        bounds = [None] * world
        dist.all_gather_object(bounds, (lo, hi))
        assert bounds[0][0] == 0 and bounds[-1][1] == TOTAL
        assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
        # every rank computes the owner of its rows' dyadic sources/consumers; all must agree
        mine = {}
        for d in (1, 2, 64, 256, TOTAL // world, TOTAL // 2):
            for pos in (lo, lo + 1, hi - 1):
                for other in (pos - d, pos + d):
                    if 0 <= other < TOTAL:
                        mine[(pos, other)] = owner_of(other, TOTAL, world)
        views = [None] * world
        dist.all_gather_object(views, mine)
        merged = {}
        for view in views:
            for key, owner in view.items():
                assert merged.setdefault(key, owner) == owner
                lo_o, hi_o = bounds[owner]
                assert lo_o <= key[1] < hi_o
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_plan_agrees():
    mp.spawn(_worker, args=(2, _port()), nprocs=2, join=True)


def test_shard_bounds_validation():
    import pytest

    with pytest.raises(ValueError):
        shard_bounds(10, 3, 0)
    with pytest.raises(ValueError):
        owner_of(10, 10, 2)
    assert torch.tensor([shard_bounds(8, 4, r)[0] for r in range(4)]).tolist() == [0, 2, 4, 6]


def test_shard_link_model_counts_remote_rows():
    """The NVLink byte model of the config-5 bench line equals a row-by-row count: far K/V
    sources on other ranks (forward and backward) and far consumers past the shard end
    (backward: their Q, dO, K, V and LSE)."""
    import bench
    from sbda_b200 import sbda_layer_offsets

    total, heads, dim, elem = 2048, 2, 16, 2
    for world in (1, 2, 4, 8):
        shard = total // world
        layers = sbda_layer_offsets(11)
        model = bench.shard_link_model(total, world, heads, dim, elem, layers, hbm_gbs=1.0, link_gbs=1.0)
        worst, target = 0, 0.0
        local = shard * heads * (11 * dim * elem + 8)
        for offsets in layers:
            d = max(offsets)
            bound = local
            for rank in range(world):
                lo, hi = shard_bounds(total, world, rank)
                remote = 0
                if d >= 3:
                    for i in range(lo, hi):
                        if 0 <= i - d < lo:
                            remote += 2 * heads * 2 * dim * elem
                        if hi <= i + d < total:
                            remote += heads * (4 * dim * elem + 4)
                worst = max(worst, remote)
                bound = max(bound, remote)
            target += bound
        assert model["max_remote_bytes_one_layer"] == worst
        assert abs(model["target_ms"] - target * 1e-6) < 1e-9 * target


def test_sharded_forward_needs_a_preallocated_lse():
    """``sharded_forward`` never allocates symmetric memory itself (an allocation there would be a
    collective and a buffer the group keeps): without ``lse`` it raises before any work."""
    import pytest

    from sbda_b200.sharded import sharded_forward

    q = torch.zeros(1, 2, 64, 16)
    with pytest.raises(ValueError, match="lse"):
        sharded_forward(q, q, q, (0, 1), shards=None)
