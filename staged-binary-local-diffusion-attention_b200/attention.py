"""``BinaryPathAttention`` / ``SBDAttention`` drop-in modules on the B200 kernels.

Same constructors, state-dict keys (``q, k, v, out, q_norm.weight,
k_norm.weight``) and ``forward`` signature as the reference modules
(``BiAttn/left_v2.py:100-198, 413-438``): ``BinaryPathAttention`` takes any
path topology, ``SBDAttention`` is its ``topology="sbda"`` subclass.  The fused route of the reference
(``left_v2.py:263-306``) serves the plain case; padding masks with interior
holes, ``seam_reset`` and caller path tables (``path_indices``/``path_valid``,
up to four sources per row) -- which the reference sends to its eager path --
run on the B200 kernels with a per-row source mask (``source_mask`` /
``path_source_mask`` below).  CPU tensors raise instead of silently running
another implementation.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from .norm_rope import norm_rope, normed_attention, normed_supported
from .ops import _SBDAFunction, _SBDAPathFunction, _check_inputs
from .topology import PATH_TOPOLOGIES, topology_offsets


class HeadRMSNorm(nn.Module):
    """Holds the per-head RMSNorm weight (``attention_common.py:64-76``).

    ``forward`` is the eager formula, kept for callers that use the norm on
    its own; ``SBDAttention`` applies norm and RoPE through ``norm_rope``.
    """

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        normalized = x.float() * torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (normalized * self.weight).to(dtype=x.dtype)


class BinaryPathAttention(nn.Module):
    """Causal exact-token attention over a selectable path topology (``left_v2.py:100-198``).

    ``use_sdpa``, ``use_fused`` and ``backward_mode`` are accepted for
    signature compatibility; every mode runs the same deterministic
    gather-form kernels.  ``use_fused=False`` is refused: the exact eager route
    is the reference's, not this package's.  Layers whose topology has more
    than four sources raise ``ValueError`` in ``forward``, as the reference's
    fused ops do (``sbda_triton.py:1300-1302``).
    """

    def __init__(self, dim: int, heads: int, layer: int, *, kv_heads: int | None = None,
                 rope_theta: float = 1_000_000.0, topology: str = "binary", total_layers: int = 12,
                 use_sdpa: bool = True, use_fused: bool = True, backward_mode: str = "token") -> None:
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
            raise ValueError("the B200 attention modules only run the fused route (use_fused=True)")
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
        # True: run q/k RMSNorm + RoPE inside the attention kernels where they serve the layer
        # (head_dim 64, MHA, no source mask).  False (default): the separate norm + RoPE kernels
        # then the attention kernels, the faster route measured on B200 at 1M positions x 20
        # layers x 4 heads (50.9 vs 56.1 ms per forward + backward step).
        self.fused_norm_rope = False

    def forward(self, x: Tensor, valid_mask: Tensor | None = None, seam_reset: Tensor | None = None,
                path_indices: Tensor | None = None, path_valid: Tensor | None = None) -> Tensor:
        out = self._attend(x, valid_mask, seam_reset, path_indices, path_valid)
        if valid_mask is not None:
            out = out * valid_mask[:, :, None].to(dtype=out.dtype)
        return out

    def _attend(self, x: Tensor, valid_mask: Tensor | None = None, seam_reset: Tensor | None = None,
                path_indices: Tensor | None = None, path_valid: Tensor | None = None) -> Tensor:
        """``forward`` without the final padding-row multiply (a caller that fuses it, the
        block, applies it)."""
        if x.ndim != 3:
            raise ValueError("x must have shape [batch, sequence, dim]")
        batch, length, dim = x.shape
        if dim != self.dim:
            raise ValueError(f"expected dim={self.dim}, got {dim}")
        if valid_mask is not None and (valid_mask.shape != (batch, length) or valid_mask.dtype != torch.bool):
            raise ValueError("valid_mask must be bool with input shape")
        if seam_reset is not None and (seam_reset.shape != (batch, length) or seam_reset.dtype != torch.bool):
            raise ValueError("seam_reset must be bool with input shape")
        if path_indices is not None:  # the reference's checks, left_v2.py:212-231
            if path_indices.ndim != 3 or path_indices.shape[:2] != (batch, length):
                raise ValueError("path_indices must have shape [batch, sequence, source_count]")
            if path_indices.dtype != torch.long:
                raise ValueError("path_indices must use torch.long")
            if path_indices.device != x.device:
                raise ValueError("path_indices must be on the same device as x")
            if path_valid is None:
                path_valid = torch.ones_like(path_indices, dtype=torch.bool)
            elif (path_valid.shape != path_indices.shape or path_valid.dtype != torch.bool
                  or path_valid.device != x.device):
                raise ValueError("path_valid must match path_indices as a bool tensor")
            if path_indices.numel() and (int(path_indices.min()) < 0 or int(path_indices.max()) >= length):
                raise ValueError("path_indices contains an out-of-range source")
            if not 1 <= path_indices.shape[-1] <= 4:
                raise ValueError("the B200 path-table kernels take one to four sources per row")
        elif path_valid is not None:
            raise ValueError("path_valid needs path_indices")
        if not x.is_cuda:
            raise RuntimeError("the B200 SBDA module requires CUDA inputs")
        if path_indices is not None:
            mask = self.path_source_mask(path_indices, path_valid, valid_mask, seam_reset)
        else:
            # A prefix mask (left_v2.py:258-262) never hides a source from a valid row
            # (sources are earlier positions), so it only needs the output multiply.
            holes = (valid_mask is not None and valid_mask.shape[1] >= 2
                     and not bool(torch.all(~valid_mask[:, 1:] | valid_mask[:, :-1])))
            mask = self.source_mask(valid_mask, seam_reset) if holes or seam_reset is not None else None
        q = self.q(x).view(batch, length, self.heads, self.head_dim)
        k = self.k(x).view(batch, length, self.kv_heads, self.head_dim)
        v = self.v(x).view(batch, length, self.kv_heads, self.head_dim)
        if self.fused_norm_rope and path_indices is None and mask is None and self.kv_heads == self.heads:
            qp, kp, vp = (t.permute(0, 2, 1, 3) for t in (q, k, v))
            if normed_supported(qp, kp, vp, self.offsets):
                # One kernel each way: norm + RoPE of q/k inside the attention kernels.
                attended = normed_attention(qp, kp, vp, self.q_norm.weight, self.k_norm.weight, self.offsets,
                                            theta=self.rope_theta, q_eps=self.q_norm.eps, k_eps=self.k_norm.eps)
                return self.out(attended.transpose(1, 2).reshape(batch, length, dim))
        # RMSNorm + RoPE on the B200 kernels (attention_common.py:25-76 semantics).
        q = norm_rope(q, self.q_norm.weight, theta=self.rope_theta, eps=self.q_norm.eps)
        k = norm_rope(k, self.k_norm.weight, theta=self.rope_theta, eps=self.k_norm.eps)
        q = q.permute(0, 2, 1, 3)
        k = k.permute(0, 2, 1, 3)
        v = v.permute(0, 2, 1, 3)
        if path_indices is not None:
            _check_inputs(q, k, v, (0,), gqa=self.kv_heads != self.heads, source_counts=(1,))
            attended = _SBDAPathFunction.apply(q, k, v, path_indices.to(torch.int32).contiguous(), mask)
        else:
            _check_inputs(q, k, v, self.offsets, gqa=self.kv_heads != self.heads, source_counts=(1, 2, 3, 4))
            attended = _SBDAFunction.apply(q, k, v, self.offsets, mask)
        attended = attended.transpose(1, 2).reshape(batch, length, dim)
        return self.out(attended)

    def path_source_mask(self, path_indices: Tensor, path_valid: Tensor, valid_mask: Tensor | None,
                         seam_reset: Tensor | None) -> Tensor:
        """Source bits (uint8 ``[B, L]``) of a caller path table, ``left_v2.py:340-373``: a
        source is usable if ``path_valid`` says so, it is not after the row, and (with the
        masks) it is not padding and lies in the row's segment; padded rows keep source 0."""
        batch, length, sources = path_indices.shape
        positions = torch.arange(length, device=path_indices.device)
        usable = path_valid & (path_indices <= positions[None, :, None])
        if valid_mask is not None:
            usable = usable & torch.gather(valid_mask, 1, path_indices.reshape(batch, -1)).view_as(usable)
        if seam_reset is not None:
            segment = seam_reset.to(torch.int64).cumsum(dim=1)
            source_segment = torch.gather(segment, 1, path_indices.reshape(batch, -1)).view_as(usable)
            usable = usable & (source_segment == segment[:, :, None])
        if valid_mask is not None:
            usable = usable.clone()
            usable[:, :, 0] |= ~valid_mask
        weights = (1 << torch.arange(sources, device=path_indices.device)).to(torch.uint8)
        return (usable.to(torch.uint8) * weights).sum(dim=-1).to(torch.uint8).contiguous()

    def source_mask(self, valid_mask: Tensor | None, seam_reset: Tensor | None) -> Tensor:
        """Per-row source bits (uint8 ``[B, L]``, bit s = source s usable), ``left_v2.py:349-373``.

        Source s of row i is position ``i - o_s``: usable if it exists, is not padding,
        and lies in row i's segment (segments restart where ``seam_reset`` is set).
        Padded rows keep source 0, as in the reference; their outputs are zeroed by the
        output mask either way.
        """
        ref = valid_mask if valid_mask is not None else seam_reset
        batch, length = ref.shape
        device = ref.device
        positions = torch.arange(length, device=device)
        offsets = torch.tensor(self.offsets, device=device)
        sources = positions[:, None] - offsets[None, :]                       # [L, S]
        usable = (sources >= 0)[None].expand(batch, -1, -1)                   # [B, L, S]
        index = sources.clamp_min(0)
        if valid_mask is not None:
            usable = usable & valid_mask[:, index]
        if seam_reset is not None:
            segment = seam_reset.to(torch.int64).cumsum(dim=1)
            usable = usable & (segment[:, index] == segment[:, :, None])
        if valid_mask is not None:
            usable = usable.clone()
            usable[:, :, 0] |= ~valid_mask
        weights = (1 << torch.arange(len(self.offsets), device=device)).to(torch.uint8)
        return (usable.to(torch.uint8) * weights).sum(dim=-1).to(torch.uint8).contiguous()


class SBDAttention(BinaryPathAttention):
    """Staged Binary-Local Diffusion Attention: the ``sbda`` topology (``left_v2.py:413-438``)."""

    def __init__(self, dim: int, heads: int, layer: int, *, kv_heads: int | None = None,
                 rope_theta: float = 1_000_000.0, total_layers: int = 12, use_sdpa: bool = True,
                 use_fused: bool = True, backward_mode: str = "key") -> None:
        super().__init__(dim, heads, layer, kv_heads=kv_heads, rope_theta=rope_theta, topology="sbda",
                         total_layers=total_layers, use_sdpa=use_sdpa, use_fused=use_fused,
                         backward_mode=backward_mode)


SBDAAttention = SBDAttention
