"""The reference block around the attention op, with its elementwise parts fused.

``BiAttnBlock`` mirrors ``BiAttn/model.py:248-335`` for the attention backends
this package serves (``sbda`` and ``left_v2``) and the dense SwiGLU
feed-forward: same constructor ``(config, layer_index)``, submodule names and
state-dict keys (``norm1``, ``attn.*``, ``norm2``, ``ff.gate/up/down``).  The
reference runs norm, residual, mask and SwiGLU gate as separate eager ops
(``model.py:25-29, 58-59, 323-335``); here they are two fused kernels
(``csrc/sbda_block.cu``):

* ``rms_norm`` / ``add_rms_norm``: ``x1 = x + m * a`` (padding-row mask ``m``)
  and ``RMSNorm(x1)`` in one pass, with a deterministic backward;
* ``silu_mul``: ``silu(gate) * up``.

The GEMMs stay in cuBLAS (``nn.Linear``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import _lib
from .attention import BinaryPathAttention, SBDAttention
from .ops import _DTYPES


def _dense(t: Tensor) -> Tensor:
    """Contiguous and 16-byte aligned (the kernels' vector loads)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _check(x: Tensor, weight: Tensor) -> None:
    if not x.is_cuda:
        raise RuntimeError("the B200 block kernels require CUDA tensors")
    if x.dtype not in _DTYPES:
        raise TypeError("unsupported dtype for the B200 block kernels")
    dim = x.shape[-1]
    if dim % 8 or dim > 2048 or weight.shape != (dim,):
        raise ValueError("RMSNorm width must be a multiple of 8, at most 2048, and match the weight")


def _row_mask(mask: Tensor | None, rows: int) -> Tensor | None:
    if mask is None:
        return None
    if mask.numel() != rows:
        raise ValueError("row mask must have one entry per row")
    return mask.reshape(rows).to(torch.uint8).contiguous()


def _norm_forward(x: Tensor, add: Tensor | None, row_mask: Tensor | None, weight: Tensor, eps: float):
    dim = x.shape[-1]
    rows = x.numel() // dim
    y = torch.empty_like(x)
    x1 = torch.empty_like(x) if add is not None else None
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    w32 = weight.detach().to(torch.float32).contiguous()
    lib = _lib.load()
    with torch.cuda.device(x.device):
        status = lib.sbda_b200_rms_norm_forward(
            _DTYPES[x.dtype], rows, dim, x.data_ptr(), None if add is None else add.data_ptr(),
            None if row_mask is None else row_mask.data_ptr(), w32.data_ptr(), float(eps),
            None if x1 is None else x1.data_ptr(), y.data_ptr(), rstd.data_ptr(),
            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.raise_for_status(status, "sbda_b200_rms_norm_forward")
    return x1, y, rstd, w32


def _norm_backward(x1: Tensor, rstd: Tensor, w32: Tensor, grad_y: Tensor, grad_x1: Tensor | None,
                   row_mask: Tensor | None, with_residual: bool):
    dim = x1.shape[-1]
    rows = x1.numel() // dim
    grad_y = _dense(grad_y.to(x1.dtype))
    grad_x1 = None if grad_x1 is None else _dense(grad_x1.to(x1.dtype))
    grad_x = torch.empty_like(x1)
    grad_add = torch.empty_like(x1) if with_residual else None
    grad_w = torch.empty(dim, device=x1.device, dtype=torch.float32)
    lib = _lib.load()
    workspace = torch.empty(lib.sbda_b200_rms_norm_workspace_floats(rows, dim), device=x1.device,
                            dtype=torch.float32)
    with torch.cuda.device(x1.device):
        status = lib.sbda_b200_rms_norm_backward(
            _DTYPES[x1.dtype], rows, dim, x1.data_ptr(), rstd.data_ptr(), w32.data_ptr(), grad_y.data_ptr(),
            None if grad_x1 is None else grad_x1.data_ptr(), None if row_mask is None else row_mask.data_ptr(),
            grad_x.data_ptr(), None if grad_add is None else grad_add.data_ptr(), grad_w.data_ptr(),
            workspace.data_ptr(), workspace.numel(), torch.cuda.current_stream(x1.device).cuda_stream)
    _lib.raise_for_status(status, "sbda_b200_rms_norm_backward")
    return grad_x, grad_add, grad_w


class _RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, eps: float) -> Tensor:
        _, y, rstd, w32 = _norm_forward(x, None, None, weight, eps)
        ctx.save_for_backward(x, rstd, w32)
        ctx.weight_dtype = weight.dtype
        return y

    @staticmethod
    def backward(ctx, grad_y: Tensor):
        x, rstd, w32 = ctx.saved_tensors
        grad_x, _, grad_w = _norm_backward(x, rstd, w32, grad_y, None, None, False)
        return grad_x, grad_w.to(ctx.weight_dtype), None


class _AddRMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, add: Tensor, row_mask: Tensor | None, weight: Tensor, eps: float):
        x1, y, rstd, w32 = _norm_forward(x, add, row_mask, weight, eps)
        ctx.save_for_backward(x1, rstd, w32)
        ctx.row_mask = row_mask
        ctx.weight_dtype = weight.dtype
        return x1, y

    @staticmethod
    def backward(ctx, grad_x1: Tensor | None, grad_y: Tensor | None):
        x1, rstd, w32 = ctx.saved_tensors
        if grad_y is None:
            grad_y = torch.zeros_like(x1)
        grad_x, grad_add, grad_w = _norm_backward(x1, rstd, w32, grad_y, grad_x1, ctx.row_mask, True)
        return grad_x, grad_add, None, grad_w.to(ctx.weight_dtype), None


class _SiluMulFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate: Tensor, up: Tensor) -> Tensor:
        h = torch.empty_like(gate)
        lib = _lib.load()
        with torch.cuda.device(gate.device):
            status = lib.sbda_b200_silu_mul_forward(_DTYPES[gate.dtype], gate.numel(), gate.data_ptr(),
                                                    up.data_ptr(), h.data_ptr(),
                                                    torch.cuda.current_stream(gate.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_silu_mul_forward")
        ctx.save_for_backward(gate, up)
        return h

    @staticmethod
    def backward(ctx, grad_h: Tensor):
        gate, up = ctx.saved_tensors
        grad_h = _dense(grad_h.to(gate.dtype))
        grad_gate, grad_up = torch.empty_like(gate), torch.empty_like(up)
        lib = _lib.load()
        with torch.cuda.device(gate.device):
            status = lib.sbda_b200_silu_mul_backward(
                _DTYPES[gate.dtype], gate.numel(), gate.data_ptr(), up.data_ptr(), grad_h.data_ptr(),
                grad_gate.data_ptr(), grad_up.data_ptr(), torch.cuda.current_stream(gate.device).cuda_stream)
        _lib.raise_for_status(status, "sbda_b200_silu_mul_backward")
        return grad_gate, grad_up


def rms_norm(x: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    """``F.rms_norm(x, (dim,), weight, eps)`` (``model.py:25-29``) on the fused kernel."""
    _check(x, weight)
    return _RMSNormFunction.apply(_dense(x), weight, eps)


def add_rms_norm(x: Tensor, add: Tensor, weight: Tensor, eps: float = 1e-6,
                 row_mask: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """``x1 = x + m * add`` and ``RMSNorm(x1)`` in one pass (``model.py:325-327`` with the
    attention's padding-row multiply, ``left_v2.py:404``); returns ``(x1, norm)``."""
    _check(x, weight)
    if add.shape != x.shape or add.dtype != x.dtype:
        raise ValueError("residual addend must match x")
    rows = x.numel() // x.shape[-1]
    return _AddRMSNormFunction.apply(_dense(x), _dense(add), _row_mask(row_mask, rows), weight, eps)


def silu_mul(gate: Tensor, up: Tensor) -> Tensor:
    """``F.silu(gate) * up`` (``model.py:59``) on the fused kernel."""
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError("gate and up must match")
    if not gate.is_cuda:
        raise RuntimeError("the B200 block kernels require CUDA tensors")
    if gate.dtype not in _DTYPES:
        raise TypeError("unsupported dtype for the B200 block kernels")
    if gate.numel() % 8:
        raise ValueError("silu_mul needs a multiple of 8 elements")
    return _SiluMulFunction.apply(_dense(gate), _dense(up))


class RMSNorm(nn.Module):
    """``model.py:18-29``: same constructor and ``weight`` parameter."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        return rms_norm(x, self.weight, self.eps)


class SwiGLU(nn.Module):
    """``model.py:32-59``: same constructor, hidden-width rule and ``gate/up/down`` layers."""

    def __init__(self, dim: int, ff_mult: float, dropout: float = 0.0, *, hidden_size: int | None = None,
                 bias: bool = True) -> None:
        super().__init__()
        hidden = max(64, math.ceil(dim * math.pi / 64) * 64) if hidden_size is None else hidden_size
        if hidden < 1:
            raise ValueError("SwiGLU hidden_size must be positive")
        self.hidden_size = hidden
        self.gate = nn.Linear(dim, hidden, bias=bias)
        self.up = nn.Linear(dim, hidden, bias=bias)
        self.down = nn.Linear(hidden, dim, bias=bias)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: Tensor) -> Tensor:
        return self.dropout(self.down(silu_mul(self.gate(x), self.up(x))))


class BiAttnBlock(nn.Module):
    """Pre-norm attention + SwiGLU block, ``model.py:248-335``, for the ``sbda`` and
    ``left_v2`` attention backends and the dense feed-forward."""

    def __init__(self, config, layer_index: int) -> None:
        super().__init__()
        self.layer_index = int(layer_index)
        self.norm1 = RMSNorm(config.dim)
        backend = getattr(config, "attention_backend", "sbda")
        if backend == "sbda":
            self.attn = SBDAttention(
                config.dim, config.heads, layer=layer_index + 1, kv_heads=config.kv_heads,
                rope_theta=config.rope_theta, total_layers=config.layers, use_sdpa=config.path_sdpa,
                use_fused=config.sbda_fused, backward_mode=config.sbda_backward,
            )
        elif backend == "left_v2":
            self.attn = BinaryPathAttention(
                config.dim, config.heads, layer=layer_index + 1, kv_heads=config.kv_heads,
                rope_theta=config.rope_theta, topology=config.path_topology, total_layers=config.layers,
                use_sdpa=config.path_sdpa,
            )
        else:
            raise NotImplementedError(f"attention backend {backend!r} is not served by the B200 kernels")
        self.norm2 = RMSNorm(config.dim)
        if getattr(config, "ff_mode", "dense") != "dense":
            raise NotImplementedError("only the dense SwiGLU feed-forward is served by the B200 block")
        self.ff = SwiGLU(config.dim, config.ff_mult, config.dropout, hidden_size=config.ff_hidden,
                         bias=config.ff_bias)

    def forward(self, x: Tensor, valid_mask: Tensor | None, seam_reset: Tensor | None = None,
                path_indices: Tensor | None = None, path_valid: Tensor | None = None) -> Tensor:
        normalized = self.norm1(x)
        layer_paths = None if path_indices is None else path_indices[:, self.layer_index]
        layer_valid = None if path_valid is None else path_valid[:, self.layer_index]
        attended = self.attn._attend(normalized, valid_mask, seam_reset, layer_paths, layer_valid)
        # x + mask * attended and norm2 of the sum in one pass (model.py:325-327).
        x, ff_input = add_rms_norm(x, attended, self.norm2.weight, self.norm2.eps, valid_mask)
        ff = self.ff(ff_input)
        if valid_mask is not None:
            return torch.addcmul(x, ff, valid_mask[:, :, None].to(ff.dtype))
        return x + ff
