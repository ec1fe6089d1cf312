"""Batch x head partitioning on the kernels: the ranks' pieces together equal the whole batch."""

from __future__ import annotations

import pytest
import torch

import sbda_b200
from sbda_b200.partition import partitioned_backward, partitioned_forward

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("heads,kv_heads", [(8, 8), (8, 2)])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partitioned_ranks_equal_whole_batch(world, heads, kv_heads):
    batch, length = 3, 4096
    g = torch.Generator(device="cuda").manual_seed(world + heads)

    def make(h):
        return torch.randn(batch, length, h, 64, device="cuda", generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)

    q, k, v, do = make(heads), make(kv_heads), make(kv_heads), make(heads)
    for layer in (2, 7, 12):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        ref_out, ref_lse = sbda_b200.sbda_forward(q, k, v, offsets)
        ref = sbda_b200.sbda_backward(q, k, v, do, ref_lse, offsets)
        out = torch.full_like(q, float("nan"))
        lse = torch.full((batch, heads, length), float("nan"), device="cuda")
        grads = tuple(torch.full_like(t, float("nan")) for t in (q, k, v))
        for rank in range(world):
            partitioned_forward(q, k, v, offsets, world, rank, out=out, lse=lse)
        for rank in range(world):
            partitioned_backward(q, k, v, do, lse, offsets, world, rank, grads=grads)
        assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
        for name, a, b in zip(("dQ", "dK", "dV"), grads, ref):
            assert torch.equal(a, b), f"layer {layer} world {world}: {name}"
    assert sbda_b200.device_status(reset=True) == 0
