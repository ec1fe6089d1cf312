"""Sequence-sharded SBDA (contiguous shards, dyadic halos from the owning rank).

1. Emulated ranks on one GPU: the sharded kernels see "rank r's buffer" only as an address,
   so W ranks are W slices of one sequence; one call per rank must reproduce the unsharded
   op of the same kernel family on the whole sequence.  Covers owner selection, near/far
   halos across shard ends, global-position masks and remote LSE reads for W = 2, 4, 8, on
   the windowed and the general kernels.
2. Two real ranks (two GPUs, two processes, NCCL + symmetric memory), when available.
"""

from __future__ import annotations

import ctypes
import os
import socket

import pytest
import torch

import sbda_b200
from sbda_b200 import _lib
from sbda_b200.ops import _DTYPES, _tensor_arg

pytestmark = pytest.mark.gpu


def _arr(views):
    arr = (_lib.SbdaTensor * len(views))()
    for i, t in enumerate(views):
        arr[i] = _tensor_arg(t)
    return arr


def _emulated(q, k, v, do, offsets, world):
    """Run the sharded entry points once per emulated rank; returns whole-sequence outputs."""
    lib = _lib.load()
    batch, heads, total, dim = q.shape
    ls = total // world
    sl = lambda t, r: t[:, :, r * ls:(r + 1) * ls]  # noqa: E731
    out = torch.empty_like(q)
    lse = torch.empty((world, batch, heads, ls), device=q.device, dtype=torch.float32)
    shape = _lib.SbdaShape(batch, heads, k.shape[1], ls, dim)
    offs = _lib.offsets_array(offsets)
    stream = torch.cuda.current_stream().cuda_stream
    ks, vs = _arr([sl(k, r) for r in range(world)]), _arr([sl(v, r) for r in range(world)])
    for r in range(world):
        st = lib.sbda_b200_forward_sharded_ex(sbda_b200.current_family(), _DTYPES[q.dtype], shape, offs,
                                              len(offsets), dim ** -0.5, r, world, _tensor_arg(sl(q, r)), ks, vs,
                                              _tensor_arg(sl(out, r)), lse[r].data_ptr(), stream)
        assert st == 0, _lib.status_string(st)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    qs, dos = _arr([sl(q, r) for r in range(world)]), _arr([sl(do, r) for r in range(world)])
    lses = (ctypes.c_void_p * world)(*[lse[r].data_ptr() for r in range(world)])
    for r in range(world):
        st = lib.sbda_b200_backward_sharded_ex(sbda_b200.current_family(), _DTYPES[q.dtype], shape, offs,
                                               len(offsets), dim ** -0.5, r, world, qs, ks, vs, dos, lses,
                                               _tensor_arg(sl(dq, r)), _tensor_arg(sl(dk, r)),
                                               _tensor_arg(sl(dv, r)), stream)
        assert st == 0, _lib.status_string(st)
    return out, dq, dk, dv


def _whole(q, k, v, do, offsets, path=1):
    """The unsharded kernels of family ``path`` (0 = auto, 1 = general) on the whole sequence."""
    with sbda_b200.kernel_family(path):
        out, lse = sbda_b200.sbda_forward(q, k, v, offsets)
        dq, dk, dv = sbda_b200.sbda_backward(q, k, v, do, lse, offsets)
    return out, dq, dk, dv


@pytest.mark.parametrize("path", [0, 1], ids=["windowed", "general"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_shards_match_whole_sequence(world, path):
    """Sharded calls equal the same kernel family on the whole sequence, bit for bit: the
    windowed kernels (chain walks whose far tiles, pre tiles and halos come from other shards;
    local and local-carry walks across shard ends; a far offset longer than a shard) and the
    general kernels."""
    total = 8 * 1024
    g = torch.Generator(device="cuda").manual_seed(world)
    make = lambda h: torch.randn(1, total, h, 64, device="cuda", generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)  # noqa: E731
    q, k, v, do = make(4), make(4), make(4), make(4)
    with sbda_b200.kernel_family(path):
        for layer in (1, 2, 3, 5, 6, 7, 8, 10, 11, 12, 13, 14):
            offsets = sbda_b200.topology_offsets(layer, topology="sbda")
            got = _emulated(q, k, v, do, offsets, world)
            ref = _whole(q, k, v, do, offsets, path)
            for name, a, b in zip(("O", "dQ", "dK", "dV"), got, ref):
                assert torch.equal(a, b), f"layer {layer} world {world}: {name} differs"
    assert sbda_b200.device_status(reset=True) == 0


def test_emulated_shards_gqa_and_fp32():
    total, world = 4 * 512, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(2, 4, total, 32, device="cuda", generator=g)
    k, v = (torch.randn(2, 2, total, 32, device="cuda", generator=g) for _ in range(2))
    do = torch.randn_like(q)
    for offsets in ((0, 1, 2, 128), (0, 1, 2, 512), (0, 2), (0, 1, 2, 1024)):
        got = _emulated(q, k, v, do, offsets, world)
        ref = _whole(q, k, v, do, offsets)
        for name, a, b in zip(("O", "dQ", "dK", "dV"), got, ref):
            torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6, msg=f"{offsets} {name}")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank: int, world: int, port: int, result: "torch.multiprocessing.Queue") -> None:
    import datetime

    import torch.distributed as dist

    from sbda_b200.sharded import ShardGroup, shard_bounds, sharded_backward, sharded_forward

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        shards = ShardGroup()
        total = 8192
        lo, hi = shard_bounds(total, world, rank)
        g = torch.Generator(device=dev).manual_seed(11)
        full = [torch.randn(1, total, 4, 64, device=dev, generator=g).to(torch.bfloat16) for _ in range(4)]
        bufs = [shards.empty(1, hi - lo, 4, 64, dtype=torch.bfloat16, device=dev) for _ in range(4)]
        for buf, src in zip(bufs, full):
            buf.copy_(src[:, lo:hi])
        q, k, v, do = (b.permute(0, 2, 1, 3) for b in bufs)
        lse = shards.empty(1, 4, hi - lo, dtype=torch.float32, device=dev)
        ok = True
        for layer in (3, 9, 12, 13, 14):
            offsets = sbda_b200.topology_offsets(layer, topology="sbda")
            out, _ = sharded_forward(q, k, v, offsets, shards, lse=lse)
            dq, dk, dv = sharded_backward(q, k, v, do, lse, offsets, shards)
            shards.barrier()
            whole = [t.permute(0, 2, 1, 3) for t in full]
            ref = _whole(*whole, offsets, 0)
            for a, b in zip((out, dq, dk, dv), ref):
                ok &= bool(torch.equal(a, b[:, :, lo:hi]))
        torch.cuda.synchronize()
        result.put((rank, ok, sbda_b200.device_status(reset=True)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_shards_over_nvlink():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    outcomes = sorted(result.get(timeout=5) for _ in range(2))
    for p in procs:
        assert p.exitcode == 0
    for rank, ok, fault in outcomes:
        assert ok, f"rank {rank} differs from the single-GPU result"
        assert fault == 0


def test_repeated_sharded_calls_keep_state_flat():
    """A hundred sharded forward + backward calls on a one-rank group hold no new buffers or
    handles: ``lse`` is the caller's, and nothing is registered per call."""
    from sbda_b200.sharded import ShardGroup, sharded_backward, sharded_forward

    shards = ShardGroup()
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v, do = (torch.randn(1, 4096, 4, 64, device="cuda", generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
                   for _ in range(4))
    lse = shards.empty(1, 4, 4096, dtype=torch.float32)
    out = torch.empty_like(q)
    offsets = sbda_b200.topology_offsets(9, topology="sbda")
    sharded_forward(q, k, v, offsets, shards, out=out, lse=lse)
    sharded_backward(q, k, v, do, lse, offsets, shards)
    torch.cuda.synchronize()
    handles, allocated = len(shards._handles), torch.cuda.memory_allocated()
    for _ in range(100):
        sharded_forward(q, k, v, offsets, shards, out=out, lse=lse)
        grads = sharded_backward(q, k, v, do, lse, offsets, shards)
        del grads
    torch.cuda.synchronize()
    assert len(shards._handles) == handles
    assert torch.cuda.memory_allocated() == allocated
