"""SBDA gather-softmax attention ops on B200, drop-in for ``BiAttn/sbda_triton.py``.

Public functions keep the reference's names, argument meaning and error
types:

* ``fused_sbda_key_backward(q, k, v, offsets)`` -- ``sbda_triton.py:1467-1474``
* ``fused_sbda_gqa_key_backward(q, k, v, offsets)`` -- ``sbda_triton.py:1477-1493``
* ``fused_sbda`` / ``fused_sbda_block`` / ``fused_sbda_block_full`` --
  ``sbda_triton.py:1437-1464``; the reference's three other backward
  strategies.  All of them compute the same function, so here they share the
  one deterministic gather-form backward.

``q/k/v`` are ``[B, H, L, D]`` tensors of any strides (typically the permuted
views of ``[B, L, H, D]`` projections, ``left_v2.py:240-244``); the output has
q's dtype and strides (``empty_like``, ``sbda_triton.py:1304``).  ``offsets``
is the per-layer offset vector: a tensor on any device or a sequence of ints.
A CUDA offsets tensor is copied to the host once and cached by identity and
version, since the kernel geometry is planned on the host.

The lower-level ``sbda_forward`` / ``sbda_backward`` expose the C ABI
directly (no autograd) and return / take the fp32 log-sum-exp.

``kernel_family("general")`` (a context manager) pins the kernel family of the
calls made inside it, for tests and benchmarks that compare families.  It is
context-local (``contextvars``): other threads keep the automatic choice, and
the autograd op records the family at forward time so its backward, which
runs on autograd's worker thread, uses the same family.
"""

from __future__ import annotations

import contextlib
import contextvars
import threading
from typing import Iterator, Sequence

import torch
from torch import Tensor

from . import _lib

_DTYPES = {
    torch.float32: _lib.SBDA_DTYPE_F32,
    torch.float16: _lib.SBDA_DTYPE_F16,
    torch.bfloat16: _lib.SBDA_DTYPE_BF16,
}

_family: contextvars.ContextVar[int] = contextvars.ContextVar("sbda_b200_kernel_family", default=0)


@contextlib.contextmanager
def kernel_family(family: str | int) -> Iterator[int]:
    """Pin the kernel family (``"auto"``, ``"general"``, ``"uniform"``) of the SBDA calls made
    in this context; yields the family code."""
    token = _family.set(_lib.family_code(family))
    try:
        yield _family.get()
    finally:
        _family.reset(token)


def current_family() -> int:
    """Family code of this context (0 = automatic)."""
    return _family.get()


_offset_cache: dict[int, tuple[object, int, tuple[int, ...]]] = {}
_offset_lock = threading.Lock()


def host_offsets(offsets: Tensor | Sequence[int]) -> tuple[int, ...]:
    """Offsets as a host tuple; CUDA tensors are read once per (object, version)."""
    if not isinstance(offsets, Tensor):
        return tuple(int(o) for o in offsets)
    if offsets.device.type != "cuda":
        return tuple(int(o) for o in offsets.reshape(-1).tolist())
    key = id(offsets)
    with _offset_lock:
        entry = _offset_cache.get(key)
        if entry is not None and entry[0]() is offsets and entry[1] == offsets._version:
            return entry[2]
    values = tuple(int(o) for o in offsets.reshape(-1).tolist())
    import weakref

    with _offset_lock:
        if len(_offset_cache) > 256:
            _offset_cache.clear()
        _offset_cache[key] = (weakref.ref(offsets), offsets._version, values)
    return values


def _tensor_arg(t: Tensor) -> _lib.SbdaTensor:
    sb, sh, sl, sd = t.stride()
    return _lib.SbdaTensor(t.data_ptr(), sb, sh, sl, sd)


def _shape(q: Tensor, k: Tensor) -> _lib.SbdaShape:
    batch, heads, length, head_dim = q.shape
    return _lib.SbdaShape(batch, heads, k.shape[1], length, head_dim)


def _check_inputs(q: Tensor, k: Tensor, v: Tensor, offsets: tuple[int, ...], *, gqa: bool,
                  source_counts: tuple[int, ...] = (2, 4)) -> None:
    """Argument checks with the reference's exception types (sbda_triton.py:1295-1303, 1369-1381)."""
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("SBDA B200 kernels require CUDA tensors")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must have [B,H,L,D] shapes")
    if gqa:
        if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
            raise ValueError("q/k/v sequence and head dimensions must match")
        if k.shape[1] <= 0 or q.shape[1] % k.shape[1]:
            raise ValueError("query heads must be divisible by kv heads")
    elif q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, and v must have matching [B,H,L,D] shapes")
    if len(offsets) not in source_counts:
        raise ValueError("fused SBDA supports two or four sources")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("unsupported SBDA dtype")
    if q.shape[-1] > 128:
        raise ValueError("SBDA fused kernel supports head_dim <= 128")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k and v must be on one device")


def _check_source_mask(mask: Tensor, q: Tensor) -> None:
    if mask.dtype != torch.uint8 or mask.shape != (q.shape[0], q.shape[2]) or not mask.is_contiguous():
        raise ValueError("source_mask must be a contiguous uint8 [B, L] tensor")
    if mask.device != q.device:
        raise ValueError("source_mask must be on q's device")


def sbda_forward(q: Tensor, k: Tensor, v: Tensor, offsets: Sequence[int], *,
                 scale: float | None = None, out: Tensor | None = None,
                 lse: Tensor | None = None, source_mask: Tensor | None = None,
                 family: int | None = None) -> tuple[Tensor, Tensor]:
    """Forward through the C ABI: returns ``(out, lse)``; ``lse`` is fp32 ``[B,H,L]``.

    ``source_mask`` (optional, uint8 ``[B, L]``): bit s of row i allows source s of that row
    (``sbda_b200_forward_masked``).  ``family``: kernel family code (default: this context's,
    see :func:`kernel_family`).
    """
    family = current_family() if family is None else _lib.family_code(family)
    offsets = tuple(int(o) for o in offsets)
    batch, heads, length, head_dim = q.shape
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((batch, heads, length), device=q.device, dtype=torch.float32)
    if scale is None:
        scale = head_dim ** -0.5
    lib = _lib.load()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if source_mask is None:
            status = lib.sbda_b200_forward_ex(
                family, _DTYPES[q.dtype], _shape(q, k), _lib.offsets_array(offsets), len(offsets), float(scale),
                _tensor_arg(q), _tensor_arg(k), _tensor_arg(v), _tensor_arg(out), lse.data_ptr(), stream,
            )
        else:
            _check_source_mask(source_mask, q)
            status = lib.sbda_b200_forward_masked(
                _DTYPES[q.dtype], _shape(q, k), _lib.offsets_array(offsets), len(offsets), float(scale),
                _tensor_arg(q), _tensor_arg(k), _tensor_arg(v), source_mask.data_ptr(), _tensor_arg(out),
                lse.data_ptr(), stream,
            )
    _lib.raise_for_status(status, "sbda_b200_forward")
    return out, lse


def sbda_backward(q: Tensor, k: Tensor, v: Tensor, grad_out: Tensor, lse: Tensor,
                  offsets: Sequence[int], *, scale: float | None = None,
                  grads: tuple[Tensor, Tensor, Tensor] | None = None,
                  source_mask: Tensor | None = None, family: int | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Backward through the C ABI: returns ``(dq, dk, dv)`` in the input dtype (``source_mask`` and
    ``family`` as in :func:`sbda_forward`)."""
    family = current_family() if family is None else _lib.family_code(family)
    offsets = tuple(int(o) for o in offsets)
    if grad_out.dtype != q.dtype:
        grad_out = grad_out.to(q.dtype)
    if grad_out.device != q.device:
        raise ValueError("grad_out must be on q's device")
    if lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be a contiguous fp32 [B,H,L] tensor")
    if grads is None:
        grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
    dq, dk, dv = grads
    if scale is None:
        scale = q.shape[-1] ** -0.5
    lib = _lib.load()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if source_mask is None and family == 0 and k.shape[1] != q.shape[1]:
            # Grouped-query attention: windowed kernels with per-query-head fp32 dK/dV partials
            # in a workspace, summed per kv head in a fixed order.
            workspace = torch.empty(max(4, lib.sbda_b200_backward_grouped_workspace_floats(_shape(q, k))),
                                    device=q.device, dtype=torch.float32)
            status = lib.sbda_b200_backward_grouped(
                _DTYPES[q.dtype], _shape(q, k), _lib.offsets_array(offsets), len(offsets), float(scale),
                _tensor_arg(q), _tensor_arg(k), _tensor_arg(v), _tensor_arg(grad_out), lse.data_ptr(),
                _tensor_arg(dq), _tensor_arg(dk), _tensor_arg(dv), workspace.data_ptr(), workspace.numel(), stream,
            )
        elif source_mask is None:
            status = lib.sbda_b200_backward_ex(
                family, _DTYPES[q.dtype], _shape(q, k), _lib.offsets_array(offsets), len(offsets), float(scale),
                _tensor_arg(q), _tensor_arg(k), _tensor_arg(v), _tensor_arg(grad_out), lse.data_ptr(),
                _tensor_arg(dq), _tensor_arg(dk), _tensor_arg(dv), stream,
            )
        else:
            _check_source_mask(source_mask, q)
            status = lib.sbda_b200_backward_masked(
                _DTYPES[q.dtype], _shape(q, k), _lib.offsets_array(offsets), len(offsets), float(scale),
                _tensor_arg(q), _tensor_arg(k), _tensor_arg(v), source_mask.data_ptr(), _tensor_arg(grad_out),
                lse.data_ptr(), _tensor_arg(dq), _tensor_arg(dk), _tensor_arg(dv), stream,
            )
    _lib.raise_for_status(status, "sbda_b200_backward")
    return dq, dk, dv


class _SBDAFunction(torch.autograd.Function):
    """Autograd op: forward saves ``q, k, v, lse``; backward returns ``(dq, dk, dv, None)``.

    Mirrors the reference's ``_FusedSBDAKeyBackward`` (``sbda_triton.py:1290-1360``)
    and ``_FusedSBDAGQAKeyBackward`` (``:1363-1434``), with a fp32 LSE per row
    saved instead of the ``[B,H,L,S]`` weight table.
    """

    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, v: Tensor, offsets: tuple[int, ...],
                source_mask: Tensor | None = None) -> Tensor:
        ctx.family = current_family()
        out, lse = sbda_forward(q, k, v, offsets, source_mask=source_mask, family=ctx.family)
        ctx.save_for_backward(q, k, v, lse)
        ctx.offsets = offsets
        ctx.source_mask = source_mask
        return out

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        q, k, v, lse = ctx.saved_tensors
        dq, dk, dv = sbda_backward(q, k, v, grad_out, lse, ctx.offsets, source_mask=ctx.source_mask,
                                   family=ctx.family)
        return dq, dk, dv, None, None


def path_key_index(index: Tensor, source_mask: Tensor) -> tuple[Tensor, Tensor]:
    """Inverse of a path table: per batch, for each key position j, the codes
    ``i * S + s`` of the (row, source) pairs whose source is j and usable, sorted by
    (j, code) so the backward sums them in a fixed order.  Returns int32
    ``(offsets [B, L + 1], entries [B, L * S])``; unused entry slots are -1."""
    batch, length, sources = index.shape
    usable = ((source_mask.to(torch.int32)[:, :, None] >> torch.arange(sources, device=index.device)) & 1).bool()
    usable &= (index >= 0) & (index < length)
    codes = torch.arange(length * sources, device=index.device, dtype=torch.int64).expand(batch, -1)
    keys = torch.where(usable.reshape(batch, -1), index.reshape(batch, -1).to(torch.int64),
                       torch.full_like(codes, length))          # unused pairs sort last
    order = torch.argsort(keys * (length * sources) + codes, dim=1)
    entries = torch.where(torch.gather(keys, 1, order) < length, order, torch.full_like(order, -1))
    counts = torch.zeros(batch, length + 1, device=index.device, dtype=torch.int64)
    counts.scatter_add_(1, keys, torch.ones_like(keys))
    offsets = torch.zeros(batch, length + 1, device=index.device, dtype=torch.int64)
    offsets[:, 1:] = torch.cumsum(counts[:, :length], dim=1)
    return offsets.to(torch.int32).contiguous(), entries.to(torch.int32).contiguous()


class _SBDAPathFunction(torch.autograd.Function):
    """Attention over a caller path table (``left_v2.py:323-396``): ``index`` int32
    ``[B, L, S]``, ``source_mask`` uint8 ``[B, L]`` (bit s = source s usable)."""

    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, v: Tensor, index: Tensor, source_mask: Tensor) -> Tensor:
        batch, heads, length, head_dim = q.shape
        sources = index.shape[-1]
        out = torch.empty_like(q)
        lse = torch.empty((batch, heads, length), device=q.device, dtype=torch.float32)
        lib = _lib.load()
        with torch.cuda.device(q.device):
            status = lib.sbda_b200_forward_paths(
                _DTYPES[q.dtype], _shape(q, k), sources, head_dim ** -0.5, _tensor_arg(q), _tensor_arg(k),
                _tensor_arg(v), index.data_ptr(), source_mask.data_ptr(), _tensor_arg(out), lse.data_ptr(),
                torch.cuda.current_stream(q.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_forward_paths")
        ctx.save_for_backward(q, k, v, index, source_mask, lse)
        return out

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        q, k, v, index, source_mask, lse = ctx.saved_tensors
        sources = index.shape[-1]
        grad_out = grad_out.to(q.dtype).contiguous()
        if grad_out.data_ptr() % 16:
            grad_out = grad_out.clone()
        offsets, entries = path_key_index(index, source_mask)
        lib = _lib.load()
        shape = _shape(q, k)
        workspace = torch.empty(lib.sbda_b200_paths_workspace_floats(shape, sources), device=q.device,
                                dtype=torch.float32)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        with torch.cuda.device(q.device):
            status = lib.sbda_b200_backward_paths(
                _DTYPES[q.dtype], shape, sources, q.shape[-1] ** -0.5, _tensor_arg(q), _tensor_arg(k),
                _tensor_arg(v), index.data_ptr(), source_mask.data_ptr(), offsets.data_ptr(), entries.data_ptr(),
                _tensor_arg(grad_out), lse.data_ptr(), workspace.data_ptr(), workspace.numel(), _tensor_arg(dq),
                _tensor_arg(dk), _tensor_arg(dv), torch.cuda.current_stream(q.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_backward_paths")
        return dq, dk, dv, None, None


def _apply(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int], *, gqa: bool) -> Tensor:
    values = host_offsets(offsets)
    _check_inputs(q, k, v, values, gqa=gqa)
    return _SBDAFunction.apply(q, k, v, values)


def fused_sbda_key_backward(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """SBDA attention (MHA) with a deterministic gather-form backward.

    Drop-in for ``BiAttn.sbda_triton.fused_sbda_key_backward``
    (``sbda_triton.py:1467-1474``).
    """
    return _apply(q, k, v, offsets, gqa=False)


def fused_sbda_gqa_key_backward(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """SBDA attention with native GQA: ``k``/``v`` keep ``kv_heads`` heads.

    Drop-in for ``BiAttn.sbda_triton.fused_sbda_gqa_key_backward``
    (``sbda_triton.py:1477-1493``).  Unlike the reference, every head size
    up to 128 is served (the reference refuses head_dim not in 32/64/128).
    dK/dV sum over the query heads of a group inside one CTA.
    """
    return _apply(q, k, v, offsets, gqa=True)


def fused_sbda(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """``sbda_triton.py:1437-1443`` (token backward in the reference)."""
    return _apply(q, k, v, offsets, gqa=False)


def fused_sbda_block(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """``sbda_triton.py:1446-1453`` (block forward, token backward in the reference)."""
    return _apply(q, k, v, offsets, gqa=False)


def fused_sbda_block_full(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """``sbda_triton.py:1456-1464`` (vectorised block backward in the reference)."""
    return _apply(q, k, v, offsets, gqa=False)


def sbda_attention(q: Tensor, k: Tensor, v: Tensor, offsets: Tensor | Sequence[int]) -> Tensor:
    """General entry: 1..4 distinct offsets, MHA or GQA (``k``/``v`` with fewer heads).

    The reference's fused functions accept only S in (2, 4)
    (``sbda_triton.py:1300-1301``); this one serves every schedule of
    ``BiAttn/topology.py`` with at most four sources and at most one source
    beyond the kernel's near window.
    """
    values = host_offsets(offsets)
    _check_inputs(q, k, v, values, gqa=k.shape[1] != q.shape[1], source_counts=(1, 2, 3, 4))
    return _SBDAFunction.apply(q, k, v, values)


def device_status(reset: bool = True) -> int:
    """Device fault word set by the kernels instead of trapping (0 = clean)."""
    return _lib.device_status(reset)


__all__ = [
    "current_family", "kernel_family", "fused_sbda", "fused_sbda_block", "fused_sbda_block_full", "fused_sbda_key_backward",
    "fused_sbda_gqa_key_backward", "sbda_attention", "sbda_forward", "sbda_backward", "host_offsets",
    "device_status",
]
