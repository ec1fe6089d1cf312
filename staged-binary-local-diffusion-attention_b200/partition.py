"""Batch x head partitioning of SBDA attention across the GPUs of a data-parallel job.

Every (batch, head) sequence of an SBDA layer is independent of the others (the source schedule
only looks back along positions), so a job of B sequences x H heads splits into GPUs without
any data-path collective: rank ``r`` of ``world`` runs a contiguous range of the B * Hkv
(batch, kv head) units.  The unit is a kv head with its G = H / Hkv query heads, so a GQA group
never straddles two ranks and dK / dV need no cross-rank sum (for MHA, G = 1 and a unit is one
(batch, head) pair).  The reference runs one process on one GPU; this module is the B200 way of
spreading its batch over eight.

The helpers return views of the caller's ``[B, H, L, D]`` tensors (no copies): a rank's range is
at most three pieces -- the tail of one batch entry's heads, whole batch entries, the head of
another's -- and each piece is one strided view that the kernels take as is.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

from .ops import sbda_backward, sbda_forward


def unit_range(batch: int, kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Units ``[lo, hi)`` of ``rank`` among ``batch * kv_heads`` (batch-major) units: contiguous,
    sizes differing by at most one, the larger ones first."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if batch < 0 or kv_heads < 1:
        raise ValueError("batch must be >= 0 and kv_heads >= 1")
    units = batch * kv_heads
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def unit_pieces(lo: int, hi: int, kv_heads: int) -> list[tuple[int, int, int, int]]:
    """Decompose units ``[lo, hi)`` into pieces ``(b0, b1, h0, h1)`` (kv-head ranges): a partial
    batch entry, a block of whole entries, a partial entry -- in unit order."""
    pieces: list[tuple[int, int, int, int]] = []
    u = lo
    while u < hi:
        b, h = divmod(u, kv_heads)
        if h == 0 and hi - u >= kv_heads:  # whole batch entries
            nb = (hi - u) // kv_heads
            pieces.append((b, b + nb, 0, kv_heads))
            u += nb * kv_heads
        else:
            h1 = min(kv_heads, h + (hi - u))
            pieces.append((b, b + 1, h, h1))
            u += h1 - h
    return pieces


def rank_views(tensors: Sequence[Tensor], kv_tensors: Sequence[Tensor], world: int, rank: int
               ) -> list[tuple[list[Tensor], list[Tensor]]]:
    """Per piece of ``rank``'s range: views of the query-head tensors (``[B, H, L, D]``, and
    ``[B, H, L]`` LSE-like tensors) and of the kv-head tensors (``[B, Hkv, L, D]``)."""
    ref = kv_tensors[0]
    batch, kv_heads = ref.shape[0], ref.shape[1]
    heads = tensors[0].shape[1]
    if heads % kv_heads:
        raise ValueError("query heads must be a multiple of kv heads")
    group = heads // kv_heads
    out = []
    for b0, b1, h0, h1 in unit_pieces(*unit_range(batch, kv_heads, world, rank), kv_heads):
        qv = [t[b0:b1, h0 * group:h1 * group] for t in tensors]
        kv = [t[b0:b1, h0:h1] for t in kv_tensors]
        out.append((qv, kv))
    return out


def partitioned_forward(q: Tensor, k: Tensor, v: Tensor, offsets: Sequence[int], world: int, rank: int, *,
                        out: Tensor, lse: Tensor) -> None:
    """Forward of ``rank``'s units only, into the matching rows of ``out`` (``[B, H, L, D]``) and
    ``lse`` (contiguous fp32 ``[B, H, L]``).  Other ranks' rows are left untouched."""
    for (qv, ov, lv), (kv, vv) in rank_views((q, out, lse), (k, v), world, rank):
        sbda_forward(qv, kv, vv, offsets, out=ov, lse=lv)


def partitioned_backward(q: Tensor, k: Tensor, v: Tensor, grad_out: Tensor, lse: Tensor,
                         offsets: Sequence[int], world: int, rank: int, *,
                         grads: tuple[Tensor, Tensor, Tensor]) -> None:
    """Backward of ``rank``'s units only, into the matching rows of ``grads = (dq, dk, dv)``."""
    dq, dk, dv = grads
    for (qv, dov, lv, dqv), (kv, vv, dkv, dvv) in rank_views((q, grad_out, lse, dq), (k, v, dk, dv), world, rank):
        sbda_backward(qv, kv, vv, dov, lv, offsets, grads=(dqv, dkv, dvv))


__all__ = ["partitioned_backward", "partitioned_forward", "rank_views", "unit_pieces", "unit_range"]
