"""Per-head RMSNorm + half-split RoPE on the B200 kernels (``csrc/sbda_norm_rope.cu``).

Replaces ``_HeadRMSNorm`` followed by ``_apply_rope``
(``BiAttn/attention_common.py:13-76``) as ``BinaryPathAttention.forward``
applies them to the q/k projections (``BiAttn/left_v2.py:237-239``): one
kernel per tensor forward, one backward kernel that also produces the norm
weight's gradient (deterministic: fixed-order reduction of per-CTA partials).
"""

from __future__ import annotations

import threading

import torch
from torch import Tensor

from . import _lib
from .ops import _DTYPES

_table_cache: dict[tuple, tuple[Tensor, Tensor]] = {}
_table_lock = threading.Lock()


def rope_table(length: int, head_dim: int, theta: float, dtype: torch.dtype, device: torch.device
               ) -> tuple[Tensor, Tensor]:
    """cos/sin ``[length, head_dim // 2]`` in ``dtype``, as ``attention_common.py:13-22`` forms them.

    Angles are ``float32(position) * theta ** (-arange(0, D, 2) / D)`` in fp32, cos/sin in fp32,
    then cast to ``dtype``.  Cached per (length, head_dim, theta, dtype, device): one table
    serves every layer.  Row ``p`` is position ``p``; a sequence shard starting at global
    position ``s`` passes ``table_offset=s``.
    """
    key = (length, head_dim, float(theta), dtype, device)
    with _table_lock:
        hit = _table_cache.get(key)
    if hit is not None:
        return hit
    indices = torch.arange(0, head_dim, 2, device=device, dtype=torch.float32)
    inverse = theta ** (-indices / head_dim)
    positions = torch.arange(length, device=device)
    angles = torch.outer(positions.to(torch.float32), inverse)
    table = (angles.cos().to(dtype).contiguous(), angles.sin().to(dtype).contiguous())
    with _table_lock:
        if len(_table_cache) > 16:
            _table_cache.clear()
        _table_cache[key] = table
    return table


def _bhld_arg(t: Tensor) -> _lib.SbdaTensor:
    """A [B, L, H, D] tensor described as the [B, H, L, D] view the C ABI takes."""
    sb, sl, sh, sd = t.stride()
    return _lib.SbdaTensor(t.data_ptr(), sb, sh, sl, sd)


def _shape(t: Tensor) -> _lib.SbdaShape:
    batch, length, heads, head_dim = t.shape
    return _lib.SbdaShape(batch, heads, heads, length, head_dim)


class _NormRopeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, theta: float, eps: float, table_offset: int) -> Tensor:
        if not x.is_cuda:
            raise RuntimeError("SBDA B200 kernels require CUDA tensors")
        if x.ndim != 4:
            raise ValueError("x must be [batch, sequence, heads, head_dim]")
        if x.dtype not in _DTYPES:
            raise TypeError("unsupported SBDA dtype")
        batch, length, heads, head_dim = x.shape
        if weight.shape != (head_dim,):
            raise ValueError("weight must have shape [head_dim]")
        w32 = weight.detach().to(device=x.device, dtype=torch.float32).contiguous()
        cos = sin = None
        if head_dim % 2 == 0:
            cos, sin = rope_table(table_offset + length, head_dim, theta, x.dtype, x.device)
        y = torch.empty((batch, length, heads, head_dim), device=x.device, dtype=x.dtype)
        lib = _lib.load()
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream(x.device).cuda_stream
            status = lib.sbda_b200_norm_rope_forward(
                _DTYPES[x.dtype], _shape(x), _bhld_arg(x), _bhld_arg(y), w32.data_ptr(), float(eps),
                cos.data_ptr() if cos is not None else None, sin.data_ptr() if sin is not None else None,
                int(table_offset), stream)
        _lib.raise_for_status(status, "sbda_b200_norm_rope_forward")
        ctx.save_for_backward(x, w32)
        ctx.tables = (cos, sin)
        ctx.eps, ctx.table_offset, ctx.weight_dtype = float(eps), int(table_offset), weight.dtype
        return y

    @staticmethod
    def backward(ctx, grad_y: Tensor):
        x, w32 = ctx.saved_tensors
        cos, sin = ctx.tables
        if grad_y.dtype != x.dtype:
            grad_y = grad_y.to(x.dtype)
        grad_x = torch.empty_like(x, memory_format=torch.contiguous_format)
        grad_w = torch.empty_like(w32)
        lib = _lib.load()
        shape = _shape(x)
        workspace = torch.empty(max(1, lib.sbda_b200_norm_rope_workspace_floats(shape)), device=x.device,
                                dtype=torch.float32)
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream(x.device).cuda_stream
            status = lib.sbda_b200_norm_rope_backward(
                _DTYPES[x.dtype], shape, _bhld_arg(x), _bhld_arg(grad_y), w32.data_ptr(), ctx.eps,
                cos.data_ptr() if cos is not None else None, sin.data_ptr() if sin is not None else None,
                ctx.table_offset, _bhld_arg(grad_x), grad_w.data_ptr(), workspace.data_ptr(),
                workspace.numel(), stream)
        _lib.raise_for_status(status, "sbda_b200_norm_rope_backward")
        return grad_x, grad_w.to(ctx.weight_dtype), None, None, None


def norm_rope(x: Tensor, weight: Tensor, *, theta: float = 1_000_000.0, eps: float = 1e-6,
              position_offset: int = 0) -> Tensor:
    """RMSNorm (fp32, weight, cast back) then RoPE of ``x`` ``[B, L, H, D]``; returns a new tensor.

    ``position_offset`` is the global position of ``x[:, 0]`` (0 for a whole sequence).
    """
    return _NormRopeFunction.apply(x, weight, float(theta), float(eps), int(position_offset))


# ---------------------------------------------------------------------------
# Attention with the norm + RoPE of q and k fused into the kernels
# ---------------------------------------------------------------------------


def _tensor_arg(t: Tensor) -> _lib.SbdaTensor:
    sb, sh, sl, sd = t.stride()
    return _lib.SbdaTensor(t.data_ptr(), sb, sh, sl, sd)


def _vector_view(t: Tensor) -> bool:
    """A [B, H, L, D] view the copy engine can stage: 16-byte aligned rows and strides."""
    e = t.element_size()
    if t.data_ptr() % 16 or (t.shape[-1] > 1 and t.stride(-1) != 1):
        return False
    return all(size <= 1 or (stride > 0 and stride * e % 16 == 0) for size, stride in zip(t.shape[:3], t.stride()[:3]))


def normed_supported(q_raw: Tensor, k_raw: Tensor, v: Tensor, offsets) -> bool:
    """Whether ``normed_attention`` serves these ``[B, H, L, D]`` views and offsets on the fused
    kernels: head_dim 64, MHA, copy-engine layouts, the SBDA family's source sets."""
    if not (q_raw.is_cuda and k_raw.is_cuda and v.is_cuda) or q_raw.dtype not in _DTYPES:
        return False
    if q_raw.shape != k_raw.shape or q_raw.shape != v.shape or k_raw.dtype != q_raw.dtype or v.dtype != q_raw.dtype:
        return False
    if not (_vector_view(q_raw) and _vector_view(k_raw) and _vector_view(v)):
        return False
    batch, heads, length, head_dim = q_raw.shape
    values = tuple(int(o) for o in offsets)
    shape = _lib.SbdaShape(batch, heads, heads, length, head_dim)
    return bool(_lib.load().sbda_b200_normed_supported(_DTYPES[q_raw.dtype], shape, _lib.offsets_array(values),
                                                       len(values)))


class _NormedAttentionFunction(torch.autograd.Function):
    """``attention(rope(norm(q_raw)), rope(norm(k_raw)), v)`` in one forward and one backward
    kernel: the per-head RMSNorm and RoPE of ``attention_common.py:13-76`` run inside the SBDA
    kernels' loads, and the backward applies their Jacobian to dQ and dK before writing them.
    Saves ``q_raw, k_raw, v`` and the fp32 LSE."""

    @staticmethod
    def forward(ctx, q_raw: Tensor, k_raw: Tensor, v: Tensor, q_weight: Tensor, k_weight: Tensor,
                offsets: tuple[int, ...], theta: float, q_eps: float, k_eps: float) -> Tensor:
        batch, heads, length, head_dim = q_raw.shape
        cos, sin = rope_table(length, head_dim, theta, q_raw.dtype, q_raw.device)
        wq = q_weight.detach().to(device=q_raw.device, dtype=torch.float32).contiguous()
        wk = k_weight.detach().to(device=q_raw.device, dtype=torch.float32).contiguous()
        out = torch.empty_like(q_raw)
        lse = torch.empty((batch, heads, length), device=q_raw.device, dtype=torch.float32)
        shape = _lib.SbdaShape(batch, heads, heads, length, head_dim)
        lib = _lib.load()
        with torch.cuda.device(q_raw.device):
            status = lib.sbda_b200_forward_normed(
                _DTYPES[q_raw.dtype], shape, _lib.offsets_array(offsets), len(offsets), head_dim ** -0.5,
                _tensor_arg(q_raw), _tensor_arg(k_raw), _tensor_arg(v), wq.data_ptr(), float(q_eps), wk.data_ptr(),
                float(k_eps), cos.data_ptr(), sin.data_ptr(), 0, _tensor_arg(out), lse.data_ptr(),
                torch.cuda.current_stream(q_raw.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_forward_normed")
        ctx.save_for_backward(q_raw, k_raw, v, lse, wq, wk)
        ctx.tables = (cos, sin)
        ctx.offsets = offsets
        ctx.eps = (float(q_eps), float(k_eps))
        ctx.weight_dtypes = (q_weight.dtype, k_weight.dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        q_raw, k_raw, v, lse, wq, wk = ctx.saved_tensors
        cos, sin = ctx.tables
        offsets = ctx.offsets
        if grad_out.dtype != q_raw.dtype:
            grad_out = grad_out.to(q_raw.dtype)
        if not _vector_view(grad_out):  # the copy engine stages dO: give it the projections' layout
            grad_out = grad_out.transpose(1, 2).contiguous().transpose(1, 2)
        batch, heads, length, head_dim = q_raw.shape
        shape = _lib.SbdaShape(batch, heads, heads, length, head_dim)
        lib = _lib.load()
        offs = _lib.offsets_array(offsets)
        floats = lib.sbda_b200_backward_normed_workspace_floats(_DTYPES[q_raw.dtype], shape, offs, len(offsets))
        if floats < 0:
            raise RuntimeError("sbda_b200_backward_normed: shape is not served")
        workspace = torch.empty(max(1, floats), device=q_raw.device, dtype=torch.float32)
        dq, dk, dv = torch.empty_like(q_raw), torch.empty_like(k_raw), torch.empty_like(v)
        gwq = torch.empty(head_dim, device=q_raw.device, dtype=torch.float32)
        gwk = torch.empty(head_dim, device=q_raw.device, dtype=torch.float32)
        with torch.cuda.device(q_raw.device):
            status = lib.sbda_b200_backward_normed(
                _DTYPES[q_raw.dtype], shape, offs, len(offsets), head_dim ** -0.5, _tensor_arg(q_raw),
                _tensor_arg(k_raw), _tensor_arg(v), _tensor_arg(grad_out), lse.data_ptr(), wq.data_ptr(), ctx.eps[0],
                wk.data_ptr(), ctx.eps[1], cos.data_ptr(), sin.data_ptr(), 0, _tensor_arg(dq), _tensor_arg(dk),
                _tensor_arg(dv), gwq.data_ptr(), gwk.data_ptr(), workspace.data_ptr(), workspace.numel(),
                torch.cuda.current_stream(q_raw.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_backward_normed")
        return (dq, dk, dv, gwq.to(ctx.weight_dtypes[0]), gwk.to(ctx.weight_dtypes[1]), None, None, None, None)


def normed_attention(q_raw: Tensor, k_raw: Tensor, v: Tensor, q_weight: Tensor, k_weight: Tensor, offsets, *,
                     theta: float = 1_000_000.0, q_eps: float = 1e-6, k_eps: float = 1e-6) -> Tensor:
    """SBDA attention of the raw q/k projections with their per-head RMSNorm (weights ``q_weight``,
    ``k_weight``) and RoPE applied inside the kernels.  ``q_raw, k_raw, v`` are ``[B, H, L, D]``
    views (the permuted ``[B, L, H, D]`` projections); returns the attended ``[B, H, L, D]``.
    Same function as ``norm_rope`` on q and k followed by ``fused_sbda_key_backward``; raises
    ``ValueError`` where :func:`normed_supported` is false."""
    values = tuple(int(o) for o in offsets)
    if not normed_supported(q_raw, k_raw, v, values):
        raise ValueError("normed_attention: shape, layout or offsets not served by the fused kernels")
    return _NormedAttentionFunction.apply(q_raw, k_raw, v, q_weight, k_weight, values, float(theta), float(q_eps),
                                          float(k_eps))
