"""``SBDAttention`` drop-in module running on the B200 kernels.

Same constructor, state-dict keys (``q, k, v, out, q_norm.weight,
k_norm.weight``) and ``forward`` signature as the reference module
(``BiAttn/left_v2.py:100-198, 413-438``).  The fused route of the reference
(``left_v2.py:263-306``) is the only route here: inputs outside it -- CPU
tensors, ``seam_reset``, caller path tables, masks with interior holes --
raise instead of silently running another implementation.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from .ops import _SBDAFunction, _check_inputs
from .topology import PATH_TOPOLOGIES, topology_offsets


class HeadRMSNorm(nn.Module):
    """Per-head RMSNorm in fp32 with a learned weight (``attention_common.py:64-76``)."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        normalized = x.float() * torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (normalized * self.weight).to(dtype=x.dtype)


_rope_cache: dict[tuple, tuple[Tensor, Tensor]] = {}


def rope_tables(length: int, head_dim: int, theta: float, dtype: torch.dtype, device: torch.device,
                position_offset: int = 0) -> tuple[Tensor, Tensor]:
    """cos/sin ``[1, L, 1, D]`` in ``dtype`` from fp32 angles (``attention_common.py:13-22``).

    Cached per (length, head_dim, theta, dtype, device, offset): every layer
    of a stack shares one table.
    """
    key = (length, head_dim, float(theta), dtype, device, position_offset)
    cached = _rope_cache.get(key)
    if cached is not None:
        return cached
    indices = torch.arange(0, head_dim, 2, device=device, dtype=torch.float32)
    inverse = theta ** (-indices / head_dim)
    positions = torch.arange(length, device=device) + position_offset
    angles = torch.outer(positions.to(torch.float32), inverse)
    cos = torch.cat((angles.cos(), angles.cos()), dim=-1)[None, :, None, :].to(dtype)
    sin = torch.cat((angles.sin(), angles.sin()), dim=-1)[None, :, None, :].to(dtype)
    if len(_rope_cache) > 16:
        _rope_cache.clear()
    _rope_cache[key] = (cos, sin)
    return cos, sin


def apply_rope(q: Tensor, k: Tensor, *, theta: float, position_offset: int = 0) -> tuple[Tensor, Tensor]:
    """Half-split RoPE on ``[B, L, H, D]`` (``attention_common.py:25-50``)."""
    head_dim = q.shape[-1]
    if head_dim % 2:
        return q, k
    half = head_dim // 2
    qc, qs = rope_tables(q.shape[1], head_dim, theta, q.dtype, q.device, position_offset)
    kc, ks = rope_tables(k.shape[1], head_dim, theta, k.dtype, k.device, position_offset)

    def rotate(x: Tensor) -> Tensor:
        return torch.cat((-x[..., half:], x[..., :half]), dim=-1)

    return q * qc + rotate(q) * qs, k * kc + rotate(k) * ks


class SBDAttention(nn.Module):
    """Staged Binary-Local Diffusion Attention on the B200 kernels.

    ``use_sdpa``, ``use_fused`` and ``backward_mode`` are accepted for
    signature compatibility (``left_v2.py:416-438``); every mode runs the
    same deterministic gather-form kernels.  ``use_fused=False`` is refused:
    the exact eager route is the reference's, not this package's.
    """

    def __init__(self, dim: int, heads: int, layer: int, *, kv_heads: int | None = None,
                 rope_theta: float = 1_000_000.0, total_layers: int = 12, use_sdpa: bool = True,
                 use_fused: bool = True, backward_mode: str = "key", topology: str = "sbda") -> None:
        super().__init__()
        if dim <= 0 or heads <= 0 or dim % heads:
            raise ValueError("dim must be positive, heads must be positive, and divide dim")
        if layer < 1:
            raise ValueError("layer must be positive")
        if backward_mode not in ("token", "block", "key"):
            raise ValueError("backward_mode must be token, block, or key")
        if topology not in PATH_TOPOLOGIES:
            raise ValueError(f"unknown path topology: {topology}")
        if not use_fused:
            raise ValueError("the B200 SBDA module only runs the fused route (use_fused=True)")
        self.dim = int(dim)
        self.heads = int(heads)
        self.layer = int(layer)
        self.total_layers = int(total_layers)
        self.use_sdpa = bool(use_sdpa)
        self.use_fused = True
        self.backward_mode = backward_mode
        self.topology = topology
        self.offsets = topology_offsets(self.layer, topology=topology, total_layers=self.total_layers)
        self.register_buffer("_fused_offsets", torch.tensor(self.offsets, dtype=torch.int32), persistent=False)
        self.kv_heads = self.heads if kv_heads is None else int(kv_heads)
        if self.kv_heads <= 0 or self.heads % self.kv_heads:
            raise ValueError("heads must be divisible by kv_heads")
        self.head_dim = self.dim // self.heads
        self.rope_theta = float(rope_theta)
        if self.rope_theta <= 0:
            raise ValueError("rope_theta must be positive")
        self.q = nn.Linear(dim, dim, bias=False)
        self.k = nn.Linear(dim, self.kv_heads * self.head_dim, bias=False)
        self.v = nn.Linear(dim, self.kv_heads * self.head_dim, bias=False)
        self.q_norm = HeadRMSNorm(self.head_dim)
        self.k_norm = HeadRMSNorm(self.head_dim)
        self.out = nn.Linear(dim, dim, bias=False)

    def forward(self, x: Tensor, valid_mask: Tensor | None = None, seam_reset: Tensor | None = None,
                path_indices: Tensor | None = None, path_valid: Tensor | None = None) -> Tensor:
        if x.ndim != 3:
            raise ValueError("x must have shape [batch, sequence, dim]")
        batch, length, dim = x.shape
        if dim != self.dim:
            raise ValueError(f"expected dim={self.dim}, got {dim}")
        if valid_mask is not None and (valid_mask.shape != (batch, length) or valid_mask.dtype != torch.bool):
            raise ValueError("valid_mask must be bool with input shape")
        if seam_reset is not None or path_indices is not None or path_valid is not None:
            raise NotImplementedError("seam_reset / path tables are not served by the B200 SBDA kernels")
        if not x.is_cuda:
            raise RuntimeError("the B200 SBDA module requires CUDA inputs")
        # Prefix-mask precondition of the fused route (left_v2.py:258-262).
        if valid_mask is not None and valid_mask.shape[1] >= 2:
            if not bool(torch.all(~valid_mask[:, 1:] | valid_mask[:, :-1])):
                raise NotImplementedError("valid_mask with interior holes is not served by the B200 SBDA kernels")
        q = self.q(x).view(batch, length, self.heads, self.head_dim)
        k = self.k(x).view(batch, length, self.kv_heads, self.head_dim)
        v = self.v(x).view(batch, length, self.kv_heads, self.head_dim)
        q = self.q_norm(q)
        k = self.k_norm(k)
        q, k = apply_rope(q, k, theta=self.rope_theta)
        q = q.permute(0, 2, 1, 3)
        k = k.permute(0, 2, 1, 3)
        v = v.permute(0, 2, 1, 3)
        _check_inputs(q, k, v, self.offsets, gqa=self.kv_heads != self.heads, source_counts=(1, 2, 3, 4))
        attended = _SBDAFunction.apply(q, k, v, self.offsets)
        attended = attended.transpose(1, 2).reshape(batch, length, dim)
        out = self.out(attended)
        if valid_mask is not None:
            out = out * valid_mask[:, :, None].to(dtype=out.dtype)
        return out


SBDAAttention = SBDAttention
