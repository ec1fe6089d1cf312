"""SBDA attention over contiguous sequence shards on several GPUs.

Rank ``r`` of a process group holds positions ``[r * L, (r + 1) * L)`` of one sequence (the
reference runs one sequence on one GPU; a single sequence of millions of positions is the case
this module scales).
A query's dyadic source ``i - d`` and a key's dyadic consumer ``j + d`` may live on another
rank: the kernels (the windowed ones for SBDA schedules, the general ones otherwise) stage those
rows per tile straight from the owning GPU's buffer over NVLink (non-multicast TMA loads of peer
memory).  One rank (world 1) runs the unsharded kernels.  The buffers peers read are allocated in
symmetric memory (``torch.distributed._symmetric_memory``) so every rank can address every
other rank's copy; NCCL / the process group is used only to exchange handles and for the
device-side barrier that orders a layer's writes before its peers' reads.

Data a peer reads: forward -- K, V; backward -- Q, K, V, dO and the forward's LSE.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .ops import _DTYPES, _tensor_arg, current_family, host_offsets


def shard_bounds(total_len: int, world: int, rank: int) -> tuple[int, int]:
    """Positions ``[start, stop)`` of ``rank``'s shard; shards are equal and contiguous."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if total_len % world:
        raise ValueError("total length must be divisible by the number of shards")
    shard = total_len // world
    return rank * shard, (rank + 1) * shard


def owner_of(position: int, total_len: int, world: int) -> int:
    """Rank holding global ``position`` (``0 <= position < total_len``)."""
    if not 0 <= position < total_len:
        raise ValueError("position outside the sequence")
    return position // (total_len // world)


class ShardGroup:
    """Symmetric buffers and peer addresses for one process group.

    Without an initialised process group it is a one-rank group on the current GPU (ordinary
    memory, no barrier), so the same code runs on one GPU.
    """

    def __init__(self, group: dist.ProcessGroup | None = None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = symm_mem
        self.single = group is None and not (dist.is_available() and dist.is_initialized())
        self.group = None if self.single else (group if group is not None else dist.group.WORLD)
        self.rank = 0 if self.single else dist.get_rank(self.group)
        self.world = 1 if self.single else dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("at most 8 sequence shards")
        self._handles: dict[int, tuple[object, int]] = {}
        self._barrier_handle = None

    def empty(self, *shape: int, dtype: torch.dtype, device: torch.device | None = None) -> Tensor:
        """A tensor every rank of the group can read (collective: all ranks call it alike)."""
        device = device or torch.device("cuda", torch.cuda.current_device())
        if self.single:  # one GPU, no process group: ordinary memory, no peers
            return torch.empty(*shape, dtype=dtype, device=device)
        t = self._symm.empty(*shape, dtype=dtype, device=device)
        handle = self._symm.rendezvous(t, self.group)
        self._handles[t.untyped_storage().data_ptr()] = (handle, t.untyped_storage().data_ptr())
        if self._barrier_handle is None:
            self._barrier_handle = handle
        return t

    def peer_pointers(self, t: Tensor) -> list[int]:
        """``t``'s address on every rank, as pointers valid in this process."""
        if self.single:
            return [t.data_ptr()]
        entry = self._handles.get(t.untyped_storage().data_ptr())
        if entry is None:
            raise ValueError("tensor was not allocated by this ShardGroup")
        handle, base = entry
        offset = t.data_ptr() - handle.buffer_ptrs[self.rank]
        return [int(ptr) + offset for ptr in handle.buffer_ptrs]

    def barrier(self, timeout_ms: int = 10_000) -> None:
        """Device-side barrier on the current stream: earlier writes on every rank are visible
        after it.  The wait is bounded (``timeout_ms``), so a rank that never arrives ends the
        wait with an error instead of holding the GPU."""
        if self.single:
            return
        if self._barrier_handle is None:
            raise RuntimeError("no symmetric buffer allocated yet")
        self._barrier_handle.barrier(channel=0, timeout_ms=int(timeout_ms))


def _rank_args(shards: ShardGroup, t: Tensor):
    """``sbda_tensor`` array describing ``t`` ([B,H,L,D] view) on every rank."""
    sb, sh, sl, sd = t.stride()
    arr = (_lib.SbdaTensor * shards.world)()
    for r, ptr in enumerate(shards.peer_pointers(t)):
        arr[r] = _lib.SbdaTensor(ptr, sb, sh, sl, sd)
    return arr


def sharded_forward(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int], shards: ShardGroup,
                    *, out: Tensor | None = None, lse: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """This rank's output rows and fp32 LSE ``[B,H,L]`` for its shard.

    ``q, k, v``: this rank's shard as ``[B, H, L, D]`` views; ``k``, ``v`` and ``lse`` must come
    from ``shards.empty`` (the backward reads every rank's LSE).  ``lse`` is required: a
    symmetric allocation is a collective, so the caller makes one per layer up front (for
    example with ``shards.empty(B, H, L, dtype=torch.float32)``) and reuses it every step.
    Issues a device-side barrier first so every rank's K/V are complete; the caller barriers
    again before overwriting K/V.
    """
    if lse is None:
        raise ValueError("sharded_forward needs a preallocated symmetric lse buffer (shards.empty)")
    values = host_offsets(offsets)
    batch, heads, length, head_dim = q.shape
    if out is None:
        out = torch.empty_like(q)
    if lse.shape != (batch, heads, length) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be a contiguous fp32 [B, H, L] tensor")
    shards.barrier()
    lib = _lib.load()
    shape = _lib.SbdaShape(batch, heads, k.shape[1], length, head_dim)
    with torch.cuda.device(q.device):
        status = lib.sbda_b200_forward_sharded_ex(
            current_family(), _DTYPES[q.dtype], shape, _lib.offsets_array(values), len(values), head_dim ** -0.5,
            shards.rank, shards.world, _tensor_arg(q), _rank_args(shards, k), _rank_args(shards, v),
            _tensor_arg(out), lse.data_ptr(), torch.cuda.current_stream(q.device).cuda_stream)
    _lib.raise_for_status(status, "sbda_b200_forward_sharded")
    return out, lse


def sharded_backward(q: Tensor, k: Tensor, v: Tensor, grad_out: Tensor, lse: Tensor,
                     offsets: Tensor | Sequence[int], shards: ShardGroup) -> tuple[Tensor, Tensor, Tensor]:
    """This rank's ``(dq, dk, dv)``; ``q, k, v, grad_out, lse`` must come from ``shards.empty``."""
    values = host_offsets(offsets)
    batch, heads, length, head_dim = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    shards.barrier()
    lib = _lib.load()
    shape = _lib.SbdaShape(batch, heads, k.shape[1], length, head_dim)
    lse_ptrs = (ctypes.c_void_p * shards.world)(*shards.peer_pointers(lse))
    with torch.cuda.device(q.device):
        status = lib.sbda_b200_backward_sharded_ex(
            current_family(), _DTYPES[q.dtype], shape, _lib.offsets_array(values), len(values), head_dim ** -0.5,
            shards.rank, shards.world, _rank_args(shards, q), _rank_args(shards, k), _rank_args(shards, v),
            _rank_args(shards, grad_out), lse_ptrs, _tensor_arg(dq), _tensor_arg(dk), _tensor_arg(dv),
            torch.cuda.current_stream(q.device).cuda_stream)
    _lib.raise_for_status(status, "sbda_b200_backward_sharded")
    return dq, dk, dv
