"""``BiAttnLM``: the reference's character LM backbone on the B200 kernels.

Drop-in for ``BiAttn/model.py`` (``BiAttnConfig`` ``model.py:154-236``, ``FactorizedTokenIO``
``model.py:120-151``, ``BiAttnLM`` ``model.py:338-502``) for the configurations whose attention
the kernels serve: ``attention_backend`` ``"sbda"`` or ``"left_v2"`` (any path topology with at
most four sources per layer) and the dense SwiGLU feed-forward.  Same dataclass fields and
defaults, same submodule names and state-dict keys (``embedding``, ``layers.{i}.*``, ``norm``,
``lm_head``, or ``token_io.*`` with factorized IO), same weight initialisation and the same
``forward_hidden`` / ``forward`` / ``next_logits`` / ``next_predictions`` / ``triangle_loss``
methods.  Blocks are ``sbda_b200.block.BiAttnBlock`` (norms, residuals and the SwiGLU gate on
fused kernels, attention on the SBDA kernels, GEMMs in cuBLAS).  Other backends (the dense and
three-track baselines) and the MoE feed-forward are outside this package: the constructor
raises ``NotImplementedError`` for them.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .block import BiAttnBlock, RMSNorm
from .topology import PATH_TOPOLOGIES

SERVED_BACKENDS = ("sbda", "left_v2")


@dataclass
class BiAttnConfig:
    """Fields and defaults of the reference's ``BiAttnConfig`` (``model.py:154-236``)."""

    vocab_size: int
    dim: int = 128
    layers: int = 12
    heads: int = 4
    kv_heads: int | None = None
    rope_theta: float = 1_000_000.0
    ff_mult: float = 2.0
    ff_hidden: int | None = None
    ff_bias: bool = False
    ff_mode: str = "dense"
    dropout: float = 0.0
    tie_embeddings: bool = True
    attention_backend: str = "left"
    path_topology: str = "binary"
    path_sdpa: bool = True
    sbda_fused: bool = True
    sbda_backward: str = "key"
    causal_right: bool = False
    attention_dim: int | None = None
    attention_stride: int = 1
    attention_grid: int | None = None
    flash_attention: bool = False
    attention_activation: str = "softmax"
    token_emb_dim: int | None = None
    embedding_rank: int = 32
    moe_experts: int = 8
    moe_top_k: int = 2

    def __post_init__(self) -> None:
        if self.attention_backend == "bidirectional" and not self.causal_right:
            warnings.warn("bidirectional attention: enabling causal_right automatically", RuntimeWarning,
                          stacklevel=2)
            self.causal_right = True

    def window_schedule(self) -> tuple[int, ...]:
        return tuple(2 ** (index + 1) for index in range(self.layers))

    def validate(self) -> None:
        """The reference's checks (``model.py:208-236``), with its messages."""
        if self.vocab_size <= 0 or self.dim <= 0 or self.layers <= 0:
            raise ValueError("vocab_size, dim, and layers must be positive")
        if self.attention_backend not in ("left", "left_v2", "sbda", "full", "bidirectional"):
            raise ValueError("attention_backend must be left, left_v2, sbda, full, or bidirectional")
        if self.attention_activation not in ("softmax", "sigmoid"):
            raise ValueError("attention_activation must be softmax or sigmoid")
        if self.path_topology not in PATH_TOPOLOGIES:
            raise ValueError(f"unknown path_topology: {self.path_topology}")
        if self.heads <= 0 or self.dim % self.heads:
            raise ValueError("dim must be divisible by heads")
        kv_heads = self.heads if self.kv_heads is None else self.kv_heads
        if kv_heads <= 0 or self.heads % kv_heads:
            raise ValueError("heads must be divisible by kv_heads")
        if self.rope_theta <= 0:
            raise ValueError("rope_theta must be positive")
        if self.ff_mult <= 0 or not 0 <= self.dropout < 1:
            raise ValueError("ff_mult must be positive and dropout in [0, 1)")
        if self.ff_mode not in ("dense", "deepseek_moe"):
            raise ValueError("ff_mode must be dense or deepseek_moe")
        if self.sbda_backward not in ("token", "block", "key"):
            raise ValueError("sbda_backward must be token, block, or key")
        if self.ff_hidden is not None and self.ff_hidden <= 0:
            raise ValueError("ff_hidden must be positive when provided")
        if self.token_emb_dim is not None and self.token_emb_dim <= 0:
            raise ValueError("token_emb_dim must be positive when provided")
        if self.embedding_rank <= 0:
            raise ValueError("embedding_rank must be positive")
        if self.moe_experts <= 0 or self.moe_top_k <= 0 or self.moe_top_k > self.moe_experts:
            raise ValueError("invalid MoE expert/top-k configuration")
        attention_dim = self.dim if self.attention_dim is None else self.attention_dim
        if attention_dim <= 0 or attention_dim % self.heads:
            raise ValueError("attention_dim must be positive and divisible by heads")
        if self.attention_stride <= 0:
            raise ValueError("attention_stride must be positive")
        if self.attention_grid is not None and self.attention_grid <= 0:
            raise ValueError("attention_grid must be positive when provided")


class FactorizedTokenIO(nn.Module):
    """Low-rank token embedding and tied output projection (``model.py:120-151``)."""

    def __init__(self, vocab_size: int, model_dim: int, token_dim: int, rank: int) -> None:
        super().__init__()
        self.token_table = nn.Embedding(vocab_size, rank)
        self.up = nn.Linear(rank, token_dim, bias=False)
        self.input_proj = nn.Linear(token_dim, model_dim, bias=False)
        self.output_proj = nn.Linear(model_dim, rank, bias=False)

    def embed(self, input_ids: Tensor) -> Tensor:
        return self.input_proj(self.up(self.token_table(input_ids)))

    def forward(self, hidden: Tensor) -> Tensor:
        # The vocabulary projection stays in fp32 (as in the reference) even under autocast.
        with torch.autocast(device_type=hidden.device.type, enabled=False):
            projected = self.output_proj(hidden.float())
            return F.linear(projected, self.token_table.weight.float())


class BiAttnLM(nn.Module):
    """Character LM backbone used with lower-triangular prefix batches (``model.py:338-502``)."""

    def __init__(self, config: BiAttnConfig) -> None:
        super().__init__()
        config.validate()
        if config.attention_backend not in SERVED_BACKENDS:
            raise NotImplementedError(
                f"attention backend {config.attention_backend!r} is not served by the B200 kernels "
                f"(served: {', '.join(SERVED_BACKENDS)})")
        if config.ff_mode != "dense":
            raise NotImplementedError("only the dense SwiGLU feed-forward is served by the B200 block")
        self.config = config
        self.factorized_io = config.token_emb_dim is not None
        if self.factorized_io:
            self.token_io = FactorizedTokenIO(config.vocab_size, config.dim, config.token_emb_dim,
                                              config.embedding_rank)
            self.embedding = None
        else:
            self.token_io = None
            self.embedding = nn.Embedding(config.vocab_size, config.dim)
        self.drop = nn.Dropout(config.dropout)
        self.layers = nn.ModuleList(BiAttnBlock(config, layer_index) for layer_index in range(config.layers))
        self.norm = RMSNorm(config.dim)
        if self.factorized_io:
            self.lm_head = self.token_io
        else:
            self.lm_head = nn.Linear(config.dim, config.vocab_size, bias=False)
            if config.tie_embeddings:
                self.lm_head.weight = self.embedding.weight
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module: nn.Module) -> None:
        """N(0, 0.02) linear and embedding weights, zero biases, unit norm weights (``model.py:369-378``)."""
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
        elif isinstance(module, RMSNorm):
            nn.init.ones_(module.weight)

    def forward_hidden(self, input_ids: Tensor, valid_mask: Optional[Tensor] = None,
                       seam_reset: Optional[Tensor] = None, path_indices: Optional[Tensor] = None,
                       path_valid: Optional[Tensor] = None, path_active: Optional[Tensor] = None) -> Tensor:
        """Final hidden states before the vocabulary projection (``model.py:380-480``), with the
        reference's argument checks and messages."""
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [batch, sequence]")
        if valid_mask is not None and (valid_mask.shape != input_ids.shape or valid_mask.dtype != torch.bool):
            raise ValueError("valid_mask must be bool with input_ids shape")
        if seam_reset is not None and (seam_reset.shape != input_ids.shape or seam_reset.dtype != torch.bool):
            raise ValueError("seam_reset must be bool with input_ids shape")
        if path_indices is not None and (
                path_indices.ndim != 4 or path_indices.shape[0] != input_ids.shape[0]
                or path_indices.shape[2] != input_ids.shape[1] or path_indices.dtype != torch.long):
            raise ValueError("path_indices must have shape [batch, layers, sequence, source_count]")
        if path_valid is not None and (path_indices is None or path_valid.shape != path_indices.shape
                                       or path_valid.dtype != torch.bool):
            raise ValueError("path_valid must match path_indices as a bool tensor")
        if path_active is not None and (
                path_indices is None or path_active.ndim != 2 or path_active.shape != path_indices.shape[:2]
                or path_active.dtype != torch.bool or path_active.device != input_ids.device):
            raise ValueError("path_active must have shape [batch, layers] and match path_indices")
        if path_indices is not None and path_indices.shape[1] != len(self.layers):
            raise ValueError("path_indices layer count must match the model")
        if path_active is not None and path_active.shape[1] != len(self.layers):
            raise ValueError("path_active layer count must match the model")
        # An all-true mask carries no information: drop it once instead of in every layer.
        if valid_mask is not None and bool(valid_mask.all()):
            valid_mask = None
        x = self.drop(self.token_io.embed(input_ids) if self.factorized_io else self.embedding(input_ids))
        for layer_index, layer in enumerate(self.layers):
            if path_active is None:
                x = layer(x, valid_mask, seam_reset, path_indices, path_valid)
                continue
            active = path_active[:, layer_index]
            if not bool(active.any()):
                continue
            if bool(active.all()):
                x = layer(x, valid_mask, seam_reset, path_indices, path_valid)
                continue
            rows = active.nonzero(as_tuple=False).flatten()
            pick = lambda t: None if t is None else t.index_select(0, rows)  # noqa: E731
            updated = layer(x.index_select(0, rows), pick(valid_mask), pick(seam_reset), pick(path_indices),
                            pick(path_valid))
            x = x.clone()
            x.index_copy_(0, rows, updated)
        return self.norm(x)

    def forward(self, input_ids: Tensor, valid_mask: Optional[Tensor] = None, seam_reset: Optional[Tensor] = None,
                path_indices: Optional[Tensor] = None, path_valid: Optional[Tensor] = None,
                path_active: Optional[Tensor] = None) -> Tensor:
        return self.lm_head(self.forward_hidden(input_ids, valid_mask, seam_reset, path_indices, path_valid,
                                                path_active))

    def next_logits(self, input_ids: Tensor, valid_mask: Tensor) -> Tensor:
        """One logit vector per triangle row, at its last valid token (``model.py:488-494``)."""
        hidden = self.forward_hidden(input_ids, valid_mask)
        lengths = valid_mask.sum(dim=1) - 1
        rows = torch.arange(input_ids.shape[0], device=input_ids.device)
        return self.lm_head(hidden[rows, lengths])

    def next_predictions(self, input_ids: Tensor, valid_mask: Tensor) -> Tensor:
        return self.next_logits(input_ids, valid_mask).argmax(dim=-1)

    def triangle_loss(self, input_ids: Tensor, valid_mask: Tensor, targets: Tensor) -> Tensor:
        if targets.ndim != 1 or targets.shape[0] != input_ids.shape[0]:
            raise ValueError("targets must contain one next token per triangle row")
        return F.cross_entropy(self.next_logits(input_ids, valid_mask), targets)


__all__ = ["BiAttnConfig", "BiAttnLM", "FactorizedTokenIO", "SERVED_BACKENDS"]
