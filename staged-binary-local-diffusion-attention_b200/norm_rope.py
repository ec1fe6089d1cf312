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
