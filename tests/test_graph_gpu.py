"""Chained launches and CUDA graphs.

The windowed kernels are launched with programmatic stream serialization: a kernel's CTAs may be
scheduled while the previous kernel on the stream drains, and wait for it before their first
global memory access.  Here every forward reads the previous layer's output as its queries and
every backward reads its forward's LSE, so a kernel that read its inputs before its predecessor
finished would see stale rows.  The eager sequence must match itself bit for bit, and a CUDA
graph of the same launches must replay to the same bits.
"""

from __future__ import annotations

import pytest
import torch

import sbda_b200
from sbda_b200 import ops

pytestmark = pytest.mark.gpu

LAYERS = (1, 2, 3, 6, 7, 9, 12)


def _setup(length=12000, heads=4, dim=64, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)

    def blhd():  # [B, L, H, D] storage viewed as [B, H, L, D]
        return torch.randn(1, length, heads, dim, device="cuda", generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)

    q, k, v, do = blhd(), blhd(), blhd(), blhd()
    offsets = [sbda_b200.topology_offsets(layer, topology="sbda") for layer in LAYERS]
    outs = [torch.empty_like(q) for _ in LAYERS]
    lses = [torch.empty(1, heads, length, device="cuda") for _ in LAYERS]
    grads = [tuple(torch.empty_like(q) for _ in range(3)) for _ in LAYERS]

    def run():
        for i, off in enumerate(offsets):
            ops.sbda_forward(q if i == 0 else outs[i - 1], k, v, off, out=outs[i], lse=lses[i])
        for i in reversed(range(len(offsets))):
            ops.sbda_backward(q if i == 0 else outs[i - 1], k, v, do, lses[i], offsets[i], grads=grads[i])

    def results():
        return [t.clone() for t in outs + lses] + [t.clone() for gr in grads for t in gr]

    def clear():
        for t in outs + lses + [t for gr in grads for t in gr]:
            t.fill_(float("nan"))

    return run, results, clear


def test_chained_launches_match_themselves_and_a_graph_replay():
    run, results, clear = _setup()
    run()
    torch.cuda.synchronize()
    first = results()
    clear()
    run()
    torch.cuda.synchronize()
    again = results()
    for a, b in zip(first, again):
        assert torch.equal(a, b)

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):  # warm the launch path on the capture stream
        run()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    clear()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    replayed = results()
    for a, b in zip(first, replayed):
        assert torch.equal(a, b)
    del graph
    assert sbda_b200.device_status(reset=True) == 0
