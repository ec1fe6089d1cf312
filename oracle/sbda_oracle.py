"""CPU oracle for SBDA sparse gather-softmax attention -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the algorithm of the
reference's exact gather path (``BiAttn/left_v2.py``) and of its helpers
(``BiAttn/attention_common.py``, ``BiAttn/topology.py``).  It is the checker
that the CUDA kernels are compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it; the product package never does.

Parity of this restatement is pinned against the reference executing its own
code: ``tests/golden/make_golden.py`` imports ``BiAttn`` from the reference
checkout, records the reference module's q/k/v after RMSNorm+RoPE, the
attended output and every gradient, and ``tests/test_oracle.py`` checks this
file against those fixtures.

Semantics restated here (per batch b, head h, query i, source s with offset
o_s, scale = D**-0.5, the value the reference computes at
``left_v2.py:388``):

  valid_s  = i - o_s >= 0                                (left_v2.py:182)
  score_s  = scale * <q_i, k_{i-o_s}>   or finfo.min      (left_v2.py:385-391)
  p        = softmax(score);  p_s = 0 where not valid      (left_v2.py:392-393)
  out_i    = sum_s p_s * v_{i-o_s}                         (left_v2.py:394-396)

The backward pass is torch autograd through the same ops, exactly as in the
reference (its exact path has no hand-written backward).
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

# ---------------------------------------------------------------------------
# Source schedule (BiAttn/topology.py)
# ---------------------------------------------------------------------------

#: Topologies whose schedule this oracle restates (subset of
#: ``topology.py:3-10``: the ones with S <= 4 sources that the kernel serves).
ORACLE_TOPOLOGIES = (
    "sbda", "h8", "h8a", "h8b", "h8c", "h8d", "h8e", "binary", "h0", "h1",
    "h7", "local_jump", "longformer_local",
)


def unique_offsets(offsets: Sequence[int]) -> tuple[int, ...]:
    """Order-preserving de-duplication of non-negative offsets.

    Follows ``BiAttn/topology.py:20-21`` (``_unique_offsets``).
    """
    seen: list[int] = []
    for offset in offsets:
        offset = int(offset)
        if offset >= 0 and offset not in seen:
            seen.append(offset)
    return tuple(seen)


def schedule_offsets(layer: int, topology: str = "sbda", total_layers: int = 12) -> tuple[int, ...]:
    """Per-layer exact left offsets, restating ``BiAttn/topology.py:24-155``.

    ``sbda``/``h8``: ``(0, 2**(l-1))`` for ``l <= 2`` else
    ``unique(0, 1, 2, 2**(l-1))`` (``topology.py:141-142``).
    """
    if layer < 1:
        raise ValueError("layer must be positive")
    if total_layers < 1:
        raise ValueError("total_layers must be positive")
    stride = 2 ** (layer - 1)
    if topology in ("sbda", "h8", "h8c"):
        return (0, stride) if layer <= 2 else unique_offsets((0, 1, 2, stride))
    if topology == "h8a":
        return (0, stride) if layer <= 2 else unique_offsets((0, 1, stride))
    if topology == "h8b":
        return (0, stride) if layer <= 2 else unique_offsets((0, 2, stride))
    if topology == "h8d":
        return (0, 1, 2, stride) if layer >= 3 and layer % 2 == 1 else (0, stride)
    if topology == "h8e":
        return (unique_offsets((0, 1, 2, stride))
                if layer > max(2, total_layers - 2) else (0, stride))
    if topology in ("binary", "h0"):
        return (0, stride)
    if topology == "h1" or topology == "local_jump":
        return unique_offsets((0, 1, 2, stride))
    if topology == "h7":
        return (0, 1, 2) if layer <= 2 else (0, stride)
    if topology == "longformer_local":
        return (0, 1, 2, 3)
    raise ValueError(f"topology not restated by the oracle: {topology}")


def sbda_stage(layer: int) -> str:
    """``BiAttn/topology.py:13-17``."""
    if layer < 1:
        raise ValueError("layer must be positive")
    return "binary" if layer <= 2 else "local_diffusion"


# ---------------------------------------------------------------------------
# Exact gather path (BiAttn/left_v2.py:313-405), default route
# ---------------------------------------------------------------------------


def path_tensors(length: int, offsets: Sequence[int]) -> tuple[Tensor, Tensor]:
    """``(indices, source_valid)`` for one layer, ``left_v2.py:172-182``."""
    positions = torch.arange(length, dtype=torch.long)
    off = torch.tensor(list(offsets), dtype=torch.long)
    indices = (positions[:, None] - off[None, :]).clamp_min(0)
    valid = positions[:, None] >= off[None, :]
    return indices, valid


def source_usable(length: int, offsets: Sequence[int], valid_mask: Tensor | None,
                  seam_reset: Tensor | None) -> Tensor:
    """``source_valid`` ``[B, L, S]`` of the reference's eager path for the default
    per-layer paths with a padding mask and/or segment resets (``left_v2.py:349-373``)."""
    ref = valid_mask if valid_mask is not None else seam_reset
    indices, base = path_tensors(length, offsets)
    batch = ref.shape[0]
    source_count = indices.shape[-1]
    gather_index = indices.unsqueeze(0).expand(batch, -1, -1)
    valid = base.unsqueeze(0).expand(batch, -1, -1).clone()
    if valid_mask is not None:
        valid &= valid_mask.unsqueeze(-1).expand(-1, -1, source_count).gather(1, gather_index)
        if seam_reset is not None:
            seg = seam_reset.to(torch.int64).cumsum(dim=1)
            valid &= seg.unsqueeze(-1).expand(-1, -1, source_count).gather(1, gather_index) == seg[:, :, None]
        valid[:, :, 0] |= ~valid_mask
    elif seam_reset is not None:
        seg = seam_reset.to(torch.int64).cumsum(dim=1)
        valid &= seg.unsqueeze(-1).expand(-1, -1, source_count).gather(1, gather_index) == seg[:, :, None]
    return valid


def path_usable(indices: Tensor, path_valid: Tensor | None, valid_mask: Tensor | None,
                seam_reset: Tensor | None) -> Tensor:
    """``source_valid`` ``[B, L, S]`` of the reference's eager path for a caller path
    table (``left_v2.py:323-373``)."""
    batch, length, source_count = indices.shape
    valid = torch.ones(length, source_count, dtype=torch.bool)[None].expand(batch, -1, -1).clone()
    if path_valid is not None:
        valid &= path_valid
    positions = torch.arange(length)
    valid &= indices <= positions[None, :, None]
    if valid_mask is not None:
        valid &= valid_mask.unsqueeze(-1).expand(-1, -1, source_count).gather(1, indices)
        if seam_reset is not None:
            seg = seam_reset.to(torch.int64).cumsum(dim=1)
            valid &= seg.unsqueeze(-1).expand(-1, -1, source_count).gather(1, indices) == seg[:, :, None]
        valid[:, :, 0] |= ~valid_mask
    elif seam_reset is not None:
        seg = seam_reset.to(torch.int64).cumsum(dim=1)
        valid &= seg.unsqueeze(-1).expand(-1, -1, source_count).gather(1, indices) == seg[:, :, None]
    return valid


def exact_attention(q: Tensor, k: Tensor, v: Tensor, offsets: Sequence[int],
                    *, use_sdpa: bool = True, usable: Tensor | None = None,
                    indices: Tensor | None = None) -> Tensor:
    """Exact SBDA attention on ``[B,H,L,D]`` tensors (any float dtype).

    Restates ``left_v2.py:335-405``: the all-valid default route, or, with
    ``usable`` (``[B, L, S]``, from :func:`source_usable`), the masked route of
    rows with padding holes or segment resets.  ``use_sdpa`` selects the
    batched-matmul form (``:380-396``) or the elementwise form (``:397-405``),
    both of which the reference keeps.
    """
    batch, heads, length, head_dim = q.shape
    if indices is None:  # the layer's fixed offsets
        indices, source_valid = path_tensors(length, offsets)
        source_count = indices.shape[-1]
        idx = indices[None, None, :, :, None].expand(batch, heads, length, source_count, head_dim)
    else:                # a caller path table [B, L, S]; `usable` is then required
        source_count = indices.shape[-1]
        idx = indices[:, None, :, :, None].expand(batch, heads, length, source_count, head_dim)
        source_valid = None
    source_k = k.unsqueeze(3).expand(batch, heads, length, source_count, head_dim).gather(2, idx)
    source_v = v.unsqueeze(3).expand(batch, heads, length, source_count, head_dim).gather(2, idx)
    invalid = ~source_valid[None, None, :, :] if usable is None else ~usable[:, None, :, :]
    if use_sdpa:
        scores = torch.matmul(q.unsqueeze(-2), source_k.transpose(-1, -2)).squeeze(-2)
    else:
        scores = (q.unsqueeze(3) * source_k).sum(dim=-1)
    scores = scores * (head_dim ** -0.5)
    scores = scores.masked_fill(invalid, torch.finfo(scores.dtype).min)
    weights = scores.softmax(dim=-1)
    weights = weights.masked_fill(invalid, 0.0)
    if use_sdpa:
        return torch.matmul(weights.unsqueeze(-2), source_v).squeeze(-2)
    return (weights.unsqueeze(-1) * source_v).sum(dim=3)


def exact_lse(q: Tensor, k: Tensor, offsets: Sequence[int]) -> Tensor:
    """Natural-log sum-exp of the valid scaled scores, ``[B,H,L]`` (fp64 math).

    Not a reference output: the reference never materialises it.  The CUDA
    forward saves it for the backward; it is checked here against the same
    scores the reference softmax normalises (``left_v2.py:385-392``).
    Rows with no valid source get ``-inf``.
    """
    batch, heads, length, head_dim = q.shape
    indices, source_valid = path_tensors(length, offsets)
    s = indices.shape[-1]
    qd, kd = q.double(), k.double()
    idx = indices[None, None, :, :, None].expand(batch, heads, length, s, head_dim)
    source_k = kd.unsqueeze(3).expand(batch, heads, length, s, head_dim).gather(2, idx)
    scores = (qd.unsqueeze(3) * source_k).sum(-1) * (head_dim ** -0.5)
    scores = scores.masked_fill(~source_valid[None, None], float("-inf"))
    return torch.logsumexp(scores, dim=-1)


def exact_attention_grads(q: Tensor, k: Tensor, v: Tensor, offsets: Sequence[int],
                          grad_out: Tensor, *, dtype: torch.dtype = torch.float32
                          ) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Forward output and ``(dq, dk, dv)`` by autograd through the exact path.

    The reference's exact path is differentiated by torch autograd
    (``left_v2.py:313-410``); this does the same in ``dtype`` on the CPU.
    """
    rq, rk, rv = (t.detach().to("cpu", dtype).requires_grad_() for t in (q, k, v))
    out = exact_attention(rq, rk, rv, offsets)
    out.backward(grad_out.detach().to("cpu", dtype))
    return out.detach(), rq.grad, rk.grad, rv.grad


def _consumer_terms(q: Tensor, k: Tensor, v: Tensor, do: Tensor, offsets: Sequence[int],
                    rows: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Softmax terms of query ``rows`` in fp64: ``(p, ds, source_index, valid)``.

    ``p[..., r, s]`` is the weight of source ``s`` of query ``rows[r]``,
    ``ds = p * (dO.v_s - sum_t p_t dO.v_t)`` its score gradient (before the
    ``scale`` factor of the score), exactly the quantities autograd forms
    through ``left_v2.py:385-396``.  Rows past the end get zero terms.
    """
    length, head_dim = q.shape[2], q.shape[3]
    off = torch.tensor(list(offsets), dtype=torch.long)
    in_range = rows < length
    rows_c = rows.clamp(max=length - 1)
    src = rows_c[:, None] - off[None, :]
    valid = (src >= 0) & in_range[:, None]
    src = src.clamp_min(0)
    qd, kd, vd, dod = (t.double() for t in (q, k, v, do))
    qr, dor = qd[:, :, rows_c], dod[:, :, rows_c]            # [B,H,R,D]
    ks, vs = kd[:, :, src], vd[:, :, src]                    # [B,H,R,S,D]
    scores = (qr.unsqueeze(3) * ks).sum(-1) * head_dim ** -0.5
    scores = scores.masked_fill(~valid, float("-inf"))
    p = torch.softmax(scores, dim=-1).nan_to_num(0.0).masked_fill(~valid, 0.0)
    dp = (dor.unsqueeze(3) * vs).sum(-1)
    ds = p * (dp - (p * dp).sum(-1, keepdim=True))
    return p, ds, src, valid


def query_rows(q: Tensor, k: Tensor, v: Tensor, do: Tensor, offsets: Sequence[int],
               rows: Tensor) -> tuple[Tensor, Tensor]:
    """Output and dQ of selected query rows (fp64), for checks at full size.

    Same function as :func:`exact_attention` and its autograd, evaluated
    only where asked, so multi-million-position runs can be spot-checked.
    """
    head_dim = q.shape[3]
    p, ds, src, _ = _consumer_terms(q, k, v, do, offsets, rows)
    vs, ks = v.double()[:, :, src], k.double()[:, :, src]
    out = (p.unsqueeze(-1) * vs).sum(3)
    dq = (ds.unsqueeze(-1) * ks).sum(3) * head_dim ** -0.5
    return out, dq


def key_rows(q: Tensor, k: Tensor, v: Tensor, do: Tensor, offsets: Sequence[int],
             keys: Tensor) -> tuple[Tensor, Tensor]:
    """dK and dV of selected key rows (fp64): key ``j`` collects from queries ``j + o``."""
    head_dim = q.shape[3]
    off = list(offsets)
    dk = torch.zeros(q.shape[0], q.shape[1], len(keys), head_dim, dtype=torch.float64)
    dv = torch.zeros_like(dk)
    length = q.shape[2]
    for s, o in enumerate(off):
        consumers = keys + o
        p, ds, _, _ = _consumer_terms(q, k, v, do, offsets, consumers)
        live = (consumers < length).to(torch.float64)
        cons = consumers.clamp(max=length - 1)
        qc, doc = q.double()[:, :, cons], do.double()[:, :, cons]
        dk += (ds[..., s] * live).unsqueeze(-1) * qc * head_dim ** -0.5
        dv += (p[..., s] * live).unsqueeze(-1) * doc
    return dk, dv


# ---------------------------------------------------------------------------
# RMSNorm + RoPE prologue (BiAttn/attention_common.py)
# ---------------------------------------------------------------------------


def head_rms_norm(x: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    """``attention_common.py:72-76``: fp32 RMSNorm, cast back to ``x.dtype``."""
    normalized = x.float() * torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps)
    return (normalized * weight).to(dtype=x.dtype)


def rope_inverse_frequencies(head_dim: int, theta: float) -> Tensor:
    """``theta ** (-arange(0, D, 2) / D)`` in fp32, ``attention_common.py:16-17``."""
    indices = torch.arange(0, head_dim, 2, dtype=torch.float32)
    return theta ** (-indices / head_dim)


def rope_cos_sin(positions: Tensor, head_dim: int, theta: float, dtype: torch.dtype
                 ) -> tuple[Tensor, Tensor]:
    """``attention_common.py:13-22``: fp32 angles, cos/sin cast to ``dtype``."""
    inverse = rope_inverse_frequencies(head_dim, theta)
    angles = torch.outer(positions.to(torch.float32), inverse)
    cos = torch.cat((angles.cos(), angles.cos()), dim=-1)[None, :, None, :].to(dtype)
    sin = torch.cat((angles.sin(), angles.sin()), dim=-1)[None, :, None, :].to(dtype)
    return cos, sin


def rotate_half(x: Tensor) -> Tensor:
    """``attention_common.py:8-10``."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(q: Tensor, k: Tensor, *, theta: float, position_offset: int = 0
               ) -> tuple[Tensor, Tensor]:
    """Half-split RoPE on ``[B,L,H,D]``, ``attention_common.py:25-50``.

    ``position_offset`` shifts the absolute positions (a sequence shard that
    starts at global position ``position_offset``); the reference always uses
    ``arange(L)``, i.e. offset 0.  Odd head sizes are left unchanged.
    """
    head_dim = q.shape[-1]
    if head_dim % 2:
        return q, k
    qpos = torch.arange(q.shape[1]) + position_offset
    kpos = torch.arange(k.shape[1]) + position_offset
    qc, qs = rope_cos_sin(qpos, head_dim, theta, q.dtype)
    kc, ks = rope_cos_sin(kpos, head_dim, theta, k.dtype)
    return q * qc + rotate_half(q) * qs, k * kc + rotate_half(k) * ks


def apply_rope_table(x: Tensor, cos_half: Tensor, sin_half: Tensor) -> Tensor:
    """RoPE of ``x`` ``[B,L,H,D]`` from explicit tables ``[L, D/2]``, computed in ``x.dtype``.

    ``attention_common.py:48``: ``x * cat(cos, cos) + rotate_half(x) * cat(sin, sin)`` with the
    tables already cast (``:20-21``).  Taking the tables as inputs lets a check use exactly the
    table a device built (CPU and CUDA ``pow``/``cos`` differ in the last bit).
    """
    if x.shape[-1] % 2:
        return x
    cos = torch.cat((cos_half, cos_half), dim=-1)[None, :, None, :].to(x.dtype)
    sin = torch.cat((sin_half, sin_half), dim=-1)[None, :, None, :].to(x.dtype)
    return x * cos + rotate_half(x) * sin


def norm_rope(q_raw: Tensor, k_raw: Tensor, q_weight: Tensor, k_weight: Tensor,
              *, theta: float = 1_000_000.0, eps: float = 1e-6,
              position_offset: int = 0) -> tuple[Tensor, Tensor]:
    """Per-head RMSNorm then RoPE, as ``left_v2.py:237-239`` applies them.

    Inputs and outputs are ``[B,L,H,D]``.
    """
    q = head_rms_norm(q_raw, q_weight, eps)
    k = head_rms_norm(k_raw, k_weight, eps)
    return apply_rope(q, k, theta=theta, position_offset=position_offset)


# ---------------------------------------------------------------------------
# Whole module, default route (BiAttn/left_v2.py:191-306)
# ---------------------------------------------------------------------------


def module_forward(x: Tensor, params: dict[str, Tensor], *, heads: int, layer: int,
                   topology: str = "sbda", total_layers: int = 12,
                   theta: float = 1_000_000.0, valid_mask: Tensor | None = None) -> Tensor:
    """``SBDAttention.forward`` for the default route (MHA).

    ``params`` holds the reference state-dict keys ``q.weight``, ``k.weight``,
    ``v.weight``, ``out.weight``, ``q_norm.weight``, ``k_norm.weight``.
    ``valid_mask`` must be a prefix mask (the fused route's precondition,
    ``left_v2.py:258-262``); masked source slots are then never read by
    valid rows and the output rows are zeroed (``left_v2.py:304-305``).
    """
    batch, length, dim = x.shape
    head_dim = dim // heads
    q = torch.nn.functional.linear(x, params["q.weight"]).view(batch, length, heads, head_dim)
    k = torch.nn.functional.linear(x, params["k.weight"]).view(batch, length, heads, head_dim)
    v = torch.nn.functional.linear(x, params["v.weight"]).view(batch, length, heads, head_dim)
    q, k = norm_rope(q, k, params["q_norm.weight"], params["k_norm.weight"], theta=theta)
    offsets = schedule_offsets(layer, topology, total_layers)
    attended = exact_attention(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3),
                               v.permute(0, 2, 1, 3), offsets)
    attended = attended.transpose(1, 2).reshape(batch, length, dim)
    out = torch.nn.functional.linear(attended, params["out.weight"])
    if valid_mask is not None:
        out = out * valid_mask[:, :, None].to(dtype=out.dtype)
    return out


# ---------------------------------------------------------------------------
# Whole LM as dense causal attention (an independent evaluation of BiAttn/model.py:248-502)
# ---------------------------------------------------------------------------


def dense_source_mask(length: int, offsets: Sequence[int], device=None) -> Tensor:
    """Boolean ``[L, L]`` attention mask of a layer: query ``i`` may attend key ``j`` iff
    ``i - j`` is one of the layer's offsets (so ``j <= i``: a causal mask thinned to the sources)."""
    pos = torch.arange(length, device=device)
    delta = pos[:, None] - pos[None, :]
    allowed = torch.zeros(length, length, dtype=torch.bool, device=device)
    for o in offsets:
        allowed |= delta == int(o)
    return allowed


def lm_forward_dense(ids: Tensor, params: dict[str, Tensor], config: dict,
                     valid_mask: Tensor | None = None) -> Tensor:
    """``BiAttnLM.forward_hidden`` (MHA, dense SwiGLU, untied or tied head) followed by the
    vocabulary head, with every attention layer evaluated as dense scaled-dot-product attention
    over the whole causal square, masked to the layer's sources.

    Same function as the reference's gather path (``left_v2.py:335-405``: softmax over the
    sources, ``D**-0.5`` scale), computed by a different algorithm -- the dense causal
    cross-check of config 1.  ``params`` holds the reference's state-dict keys; ``valid_mask``
    must be a prefix mask (``model.py:323-335`` multiplies the attention and feed-forward
    outputs by it).  Returns logits ``[B, L, vocab]``.
    """
    import torch.nn.functional as F

    dim, heads, layers = config["dim"], config["heads"], config["layers"]
    theta = float(config.get("rope_theta", 1_000_000.0))
    topology = "sbda" if config.get("attention_backend") == "sbda" else config.get("path_topology", "binary")
    batch, length = ids.shape
    head_dim = dim // heads
    mask = None if valid_mask is None or bool(valid_mask.all()) else valid_mask[:, :, None]
    x = F.embedding(ids, params["embedding.weight"])
    for i in range(layers):
        pre = f"layers.{i}."
        a = pre + "attn."
        n1 = F.rms_norm(x, (dim,), params[pre + "norm1.weight"], 1e-6)
        q = F.linear(n1, params[a + "q.weight"]).view(batch, length, heads, head_dim)
        k = F.linear(n1, params[a + "k.weight"]).view(batch, length, heads, head_dim)
        v = F.linear(n1, params[a + "v.weight"]).view(batch, length, heads, head_dim)
        q = head_rms_norm(q, params[a + "q_norm.weight"])
        k = head_rms_norm(k, params[a + "k_norm.weight"])
        if head_dim % 2 == 0:
            pos = torch.arange(length, device=ids.device)
            inv = theta ** (-torch.arange(0, head_dim, 2, device=ids.device, dtype=torch.float32) / head_dim)
            ang = torch.outer(pos.to(torch.float32), inv)
            cos = torch.cat((ang.cos(), ang.cos()), -1)[None, :, None, :].to(q.dtype)
            sin = torch.cat((ang.sin(), ang.sin()), -1)[None, :, None, :].to(q.dtype)
            q, k = q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin
        offsets = schedule_offsets(i + 1, topology, layers)
        attn_mask = dense_source_mask(length, offsets, ids.device)
        att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                             attn_mask=attn_mask)
        out = F.linear(att.transpose(1, 2).reshape(batch, length, dim), params[a + "out.weight"])
        if mask is not None:
            out = out * mask.to(out.dtype)
        x = x + out
        n2 = F.rms_norm(x, (dim,), params[pre + "norm2.weight"], 1e-6)
        f = pre + "ff."
        hidden = F.silu(F.linear(n2, params[f + "gate.weight"], params.get(f + "gate.bias"))) * \
            F.linear(n2, params[f + "up.weight"], params.get(f + "up.bias"))
        ff = F.linear(hidden, params[f + "down.weight"], params.get(f + "down.bias"))
        if mask is not None:
            ff = ff * mask.to(ff.dtype)
        x = x + ff
    h = F.rms_norm(x, (dim,), params["norm.weight"], 1e-6)
    return F.linear(h, params["lm_head.weight"])


# ---------------------------------------------------------------------------
# Byte model used by the roofline (not a reference quantity)
# ---------------------------------------------------------------------------


def algorithmic_bytes(rows: int, head_dim: int, elem_bytes: int, *, backward: bool) -> int:
    """Minimum HBM bytes for ``rows`` (batch, head, position) rows of one layer.

    Forward reads Q, K, V and writes O and a fp32 LSE: ``4*D*e + 4``.
    Backward reads Q, K, V, dO, LSE and writes dQ, dK, dV: ``7*D*e + 4``.
    """
    per = (7 if backward else 4) * head_dim * elem_bytes + 4
    return rows * per


__all__ = [
    "ORACLE_TOPOLOGIES", "unique_offsets", "schedule_offsets", "sbda_stage", "path_tensors",
    "exact_attention", "exact_lse", "exact_attention_grads", "query_rows", "key_rows", "head_rms_norm",
    "rope_inverse_frequencies", "rope_cos_sin", "rotate_half", "apply_rope", "apply_rope_table", "norm_rope",
    "module_forward", "dense_source_mask", "lm_forward_dense", "algorithmic_bytes",
]

