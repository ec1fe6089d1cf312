"""Generate golden vectors by running the reference's own SBDA code on the CPU.

Run from the repository root with the reference checkout available::

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports ``BiAttn`` from the reference, builds ``SBDAttention`` modules on
the exact (non-fused) path -- the path the reference itself takes on the CPU
(``BiAttn/left_v2.py:263-267`` requires ``x.is_cuda`` for the fused route) --
and records, for seeded inputs:

* the module input ``x``, its parameters and the module output,
* the post-RMSNorm/RoPE ``q``/``k`` and the ``v`` that reach the gather core,
  captured by wrapping ``BiAttn.left_v2._apply_rope`` (the wrapper only
  records; the reference code computes every value),
* the attended output (input of ``out``) and the gradients of every one of
  the above for a seeded upstream gradient,
* the source schedule ``topology_offsets(l, topology)`` for layers 1..24.

The output is ``tests/golden/sbda_golden.npz`` (float32, a few hundred KB),
plus ``tests/golden/path_golden.npz``: ``BinaryPathAttention`` modules of
other path topologies (module input, parameters, output, input gradient and
parameter gradients; ``PATH_CASES``), and ``tests/golden/block_golden.npz``:
whole ``BiAttnBlock`` layers (``BLOCK_CASES``).
The fixture never travels with a need for the reference: the GPU tests and
the oracle tests only read the ``.npz``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

# (name, batch, length, dim, heads, layer) -- shapes chosen to cover the
# reference's own test lengths (1, 7, 129; tests/test_model.py:49), the
# config-1 smoke shape (dim 16, 2 heads, seq 32, layers 1..3), a dyadic
# offset beyond the sequence, a merged near/far window and ragged lengths.
CASES = [
    ("cfg1_l1", 1, 32, 16, 2, 1),
    ("cfg1_l2", 1, 32, 16, 2, 2),
    ("cfg1_l3", 1, 32, 16, 2, 3),
    ("len1_l3", 1, 1, 32, 4, 3),
    ("len7_l11", 1, 7, 32, 4, 11),
    ("len129_l3", 1, 129, 80, 2, 3),
    ("b2_len17_l4", 2, 17, 32, 2, 4),
    ("b2_len150_l8", 2, 150, 32, 2, 8),
    ("len160_l7_d64", 1, 160, 64, 1, 7),
]

# (name, batch, length, dim, heads, kv_heads, layer, topology): schedules served
# by the windowed, general and uniform kernels (several far offsets), a
# three-source layer and a GQA module.
PATH_CASES = [
    ("butterfly_l8", 1, 600, 32, 2, 2, 8, "butterfly"),
    ("radix4_l4", 2, 200, 32, 2, 2, 4, "radix4"),
    ("mesh_l8", 1, 300, 48, 3, 3, 8, "mesh"),
    ("h2_l7", 1, 260, 32, 2, 2, 7, "h2"),
    ("h8a_l5", 2, 40, 32, 4, 4, 5, "h8a"),
    ("binary_l3", 1, 70, 32, 2, 2, 3, "binary"),
    ("h5_l1", 1, 30, 16, 2, 2, 1, "h5"),
    ("h6_l6", 1, 200, 32, 2, 2, 6, "h6"),
    ("butterfly_gqa_l7", 1, 300, 64, 4, 2, 7, "butterfly"),
]

# Modules with data-dependent source masks, run on the reference's eager path
# (left_v2.py:349-373): (name, batch, length, dim, heads, kv_heads, layer,
# topology, padding holes, segment resets, right padding).
MASK_CASES = [
    ("sbda_holes_l5", 2, 90, 32, 2, 2, 5, "sbda", True, False, 0),
    ("sbda_seams_l4", 2, 100, 32, 2, 2, 4, "sbda", False, True, 0),
    ("sbda_both_l6", 1, 120, 32, 2, 2, 6, "sbda", True, True, 9),
    ("butterfly_seams_l7", 1, 300, 32, 2, 2, 7, "butterfly", False, True, 0),
    ("sbda_gqa_holes_l3", 1, 80, 64, 4, 2, 3, "sbda", True, False, 5),
]

# Whole blocks (BiAttn/model.py:248-335): (name, batch, length, dim, heads,
# kv_heads, layer_index, backend, topology, ff_hidden, ff_bias, mask kind).
# Mask kinds: "none", "prefix" (right padding), "holes_seams".
BLOCK_CASES = [
    ("block_sbda_l3_prefix", 2, 48, 64, 4, None, 2, "sbda", "binary", None, False, "prefix"),
    ("block_sbda_gqa_l6_holes", 1, 100, 128, 4, 2, 5, "sbda", "binary", 192, True, "holes_seams"),
    ("block_leftv2_butterfly_l8", 1, 300, 64, 2, None, 7, "left_v2", "butterfly", None, False, "none"),
    ("block_sbda_l10", 1, 200, 64, 2, None, 9, "sbda", "binary", None, False, "none"),
]

# Modules given caller path tables (left_v2.py:212-231, 323-373), on the
# reference's eager path: (name, batch, length, dim, heads, kv_heads, sources,
# path_valid drop rate, padding holes, segment resets).  Tables are causal random
# jumps (plus the row itself as source 0).
TABLE_CASES = [
    ("table_s3", 2, 120, 32, 2, 2, 3, 0.0, False, False),
    ("table_s4_valid", 1, 200, 32, 2, 2, 4, 0.2, False, False),
    ("table_s2_holes_seams", 2, 90, 32, 2, 2, 2, 0.1, True, True),
    ("table_s3_gqa", 1, 150, 64, 4, 2, 3, 0.0, True, False),
]

TOPOLOGIES = ("sbda", "h8", "h8a", "h8b", "h8c", "h8d", "h8e", "binary", "h0", "h1",
              "h7", "local_jump", "longformer_local")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    parser.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "sbda_golden.npz"))
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from BiAttn import left_v2  # noqa: E402  (reference code)
    from BiAttn.topology import topology_offsets  # noqa: E402

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    arrays: dict[str, np.ndarray] = {}
    manifest = []
    captured: dict[str, torch.Tensor] = {}
    original_rope = left_v2._apply_rope

    def recording_rope(q, k, **kwargs):
        rq, rk = original_rope(q, k, **kwargs)
        rq.retain_grad()
        rk.retain_grad()
        captured["q"], captured["k"] = rq, rk
        return rq, rk

    left_v2._apply_rope = recording_rope
    try:
        for name, batch, length, dim, heads, layer in CASES:
            torch.manual_seed(1234 + layer * 7 + length)
            attn = left_v2.SBDAttention(dim, heads, layer, use_fused=False, total_layers=12)
            with torch.no_grad():
                attn.q_norm.weight.uniform_(0.5, 1.5)
                attn.k_norm.weight.uniform_(0.5, 1.5)
            hooks = []

            def grab_v(_module, _inputs, output):
                output.retain_grad()
                captured["v"] = output

            def grab_attended(_module, inputs):
                inputs[0].retain_grad()
                captured["attended"] = inputs[0]

            hooks.append(attn.v.register_forward_hook(grab_v))
            hooks.append(attn.out.register_forward_pre_hook(grab_attended))
            x = torch.randn(batch, length, dim, requires_grad=True)
            y = attn(x)
            grad_y = torch.randn_like(y)
            y.backward(grad_y)
            for hook in hooks:
                hook.remove()
            head_dim = dim // heads
            bhld = lambda t: t.detach().reshape(batch, length, heads, head_dim).permute(0, 2, 1, 3)  # noqa: E731
            record = {
                "x": x.detach(), "y": y.detach(), "grad_y": grad_y, "dx": x.grad,
                "q": bhld(captured["q"]), "k": bhld(captured["k"]), "v": bhld(captured["v"]),
                "o": bhld(captured["attended"]),
                "do": bhld(captured["attended"].grad),
                "dq": bhld(captured["q"].grad), "dk": bhld(captured["k"].grad),
                "dv": bhld(captured["v"].grad),
            }
            for key, param in attn.state_dict().items():
                record["param." + key] = param.detach()
            for key, param in attn.named_parameters():
                record["grad." + key] = param.grad.detach()
            for key, value in record.items():
                arrays[f"{name}/{key}"] = value.contiguous().to(torch.float32).numpy()
            offsets = list(topology_offsets(layer, topology="sbda", total_layers=12))
            manifest.append({"name": name, "batch": batch, "length": length, "dim": dim,
                             "heads": heads, "layer": layer, "offsets": offsets})
    finally:
        left_v2._apply_rope = original_rope

    schedules = {}
    for topology in TOPOLOGIES:
        schedules[topology] = [list(topology_offsets(layer, topology=topology, total_layers=12))
                               for layer in range(1, 25)]
    arrays["manifest"] = np.frombuffer(json.dumps({"cases": manifest, "schedules": schedules,
                                                   "total_layers": 12}).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(manifest)} cases, {sum(a.nbytes for a in arrays.values())} bytes")

    path_arrays: dict[str, np.ndarray] = {}
    path_manifest = []
    for name, batch, length, dim, heads, kv_heads, layer, topology in PATH_CASES:
        torch.manual_seed(4321 + layer * 11 + length)
        attn = left_v2.BinaryPathAttention(dim, heads, layer, kv_heads=kv_heads, topology=topology,
                                           total_layers=12, use_fused=False)
        with torch.no_grad():
            attn.q_norm.weight.uniform_(0.5, 1.5)
            attn.k_norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(batch, length, dim, requires_grad=True)
        y = attn(x)
        grad_y = torch.randn_like(y)
        y.backward(grad_y)
        record = {"x": x.detach(), "y": y.detach(), "grad_y": grad_y, "dx": x.grad}
        for key, param in attn.state_dict().items():
            record["param." + key] = param.detach()
        for key, param in attn.named_parameters():
            record["grad." + key] = param.grad.detach()
        for key, value in record.items():
            path_arrays[f"{name}/{key}"] = value.contiguous().to(torch.float32).numpy()
        path_manifest.append({"name": name, "batch": batch, "length": length, "dim": dim, "heads": heads,
                              "kv_heads": kv_heads, "layer": layer, "topology": topology,
                              "offsets": list(topology_offsets(layer, topology=topology, total_layers=12))})
    for name, batch, length, dim, heads, kv_heads, layer, topology, holes, seams, pad in MASK_CASES:
        gen = torch.Generator().manual_seed(777 + layer * 13 + length)
        valid_mask = torch.ones(batch, length, dtype=torch.bool)
        if holes:
            valid_mask &= torch.rand(batch, length, generator=gen) > 0.15
        if pad:
            valid_mask[:, length - pad:] = False
        seam_reset = (torch.rand(batch, length, generator=gen) < 0.05) if seams else None
        torch.manual_seed(99 + layer * 5 + length)
        attn = left_v2.BinaryPathAttention(dim, heads, layer, kv_heads=kv_heads, topology=topology,
                                           total_layers=12, use_fused=False)
        with torch.no_grad():
            attn.q_norm.weight.uniform_(0.5, 1.5)
            attn.k_norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(batch, length, dim, requires_grad=True)
        has_mask = holes or pad > 0
        y = attn(x, valid_mask=valid_mask if has_mask else None, seam_reset=seam_reset)
        grad_y = torch.randn_like(y)
        y.backward(grad_y)
        record = {"x": x.detach(), "y": y.detach(), "grad_y": grad_y, "dx": x.grad}
        if has_mask:
            record["valid_mask"] = valid_mask.to(torch.float32)
        if seam_reset is not None:
            record["seam_reset"] = seam_reset.to(torch.float32)
        for key, param in attn.state_dict().items():
            record["param." + key] = param.detach()
        for key, param in attn.named_parameters():
            record["grad." + key] = param.grad.detach()
        for key, value in record.items():
            path_arrays[f"{name}/{key}"] = value.contiguous().to(torch.float32).numpy()
        path_manifest.append({"name": name, "batch": batch, "length": length, "dim": dim, "heads": heads,
                              "kv_heads": kv_heads, "layer": layer, "topology": topology,
                              "valid_mask": has_mask, "seam_reset": seam_reset is not None,
                              "offsets": list(topology_offsets(layer, topology=topology, total_layers=12))})
    for name, batch, length, dim, heads, kv_heads, sources, drop, holes, seams in TABLE_CASES:
        gen = torch.Generator().manual_seed(555 + length + sources)
        positions = torch.arange(length)
        jumps = torch.randint(0, 64, (batch, length, sources), generator=gen)
        jumps[:, :, 0] = 0
        indices = (positions[None, :, None] - jumps).clamp_min(0)
        path_valid = torch.rand(batch, length, sources, generator=gen) >= drop
        valid_mask = (torch.rand(batch, length, generator=gen) > 0.1) if holes else None
        seam_reset = (torch.rand(batch, length, generator=gen) < 0.05) if seams else None
        torch.manual_seed(4242 + length)
        attn = left_v2.BinaryPathAttention(dim, heads, 1, kv_heads=kv_heads, topology="h4_greedy",
                                           total_layers=12, use_fused=False)
        with torch.no_grad():
            attn.q_norm.weight.uniform_(0.5, 1.5)
            attn.k_norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(batch, length, dim, requires_grad=True)
        y = attn(x, valid_mask=valid_mask, seam_reset=seam_reset, path_indices=indices, path_valid=path_valid)
        grad_y = torch.randn_like(y)
        y.backward(grad_y)
        record = {"x": x.detach(), "y": y.detach(), "grad_y": grad_y, "dx": x.grad,
                  "path_indices": indices.to(torch.float32), "path_valid": path_valid.to(torch.float32)}
        if valid_mask is not None:
            record["valid_mask"] = valid_mask.to(torch.float32)
        if seam_reset is not None:
            record["seam_reset"] = seam_reset.to(torch.float32)
        for key, param in attn.state_dict().items():
            record["param." + key] = param.detach()
        for key, param in attn.named_parameters():
            record["grad." + key] = param.grad.detach()
        for key, value in record.items():
            path_arrays[f"{name}/{key}"] = value.contiguous().to(torch.float32).numpy()
        path_manifest.append({"name": name, "batch": batch, "length": length, "dim": dim, "heads": heads,
                              "kv_heads": kv_heads, "layer": 1, "topology": "h4_greedy",
                              "valid_mask": valid_mask is not None, "seam_reset": seam_reset is not None,
                              "path_table": True,
                              "offsets": list(topology_offsets(1, topology="h4_greedy", total_layers=12))})
    path_arrays["manifest"] = np.frombuffer(json.dumps({"cases": path_manifest}).encode(), dtype=np.uint8)

    from BiAttn.model import BiAttnBlock, BiAttnConfig  # noqa: E402  (reference code)

    block_arrays: dict[str, np.ndarray] = {}
    block_manifest = []
    for name, batch, length, dim, heads, kv_heads, layer_index, backend, topology, ff_hidden, ff_bias, kind in \
            BLOCK_CASES:
        config = BiAttnConfig(vocab_size=96, dim=dim, layers=12, heads=heads, kv_heads=kv_heads,
                              ff_hidden=ff_hidden, ff_bias=ff_bias, attention_backend=backend,
                              path_topology=topology)
        torch.manual_seed(2024 + layer_index * 3 + length)
        block = BiAttnBlock(config, layer_index)
        with torch.no_grad():
            for norm in (block.norm1, block.norm2, block.attn.q_norm, block.attn.k_norm):
                norm.weight.uniform_(0.5, 1.5)
        gen = torch.Generator().manual_seed(31 + length)
        valid_mask = seam_reset = None
        if kind == "prefix":
            valid_mask = torch.ones(batch, length, dtype=torch.bool)
            valid_mask[-1, length - 7:] = False
        elif kind == "holes_seams":
            valid_mask = torch.rand(batch, length, generator=gen) > 0.12
            seam_reset = torch.rand(batch, length, generator=gen) < 0.04
        x = torch.randn(batch, length, dim, requires_grad=True)
        y = block(x, valid_mask, seam_reset)
        grad_y = torch.randn_like(y)
        y.backward(grad_y)
        record = {"x": x.detach(), "y": y.detach(), "grad_y": grad_y, "dx": x.grad}
        if valid_mask is not None:
            record["valid_mask"] = valid_mask.to(torch.float32)
        if seam_reset is not None:
            record["seam_reset"] = seam_reset.to(torch.float32)
        for key, param in block.state_dict().items():
            record["param." + key] = param.detach()
        for key, param in block.named_parameters():
            record["grad." + key] = param.grad.detach()
        for key, value in record.items():
            block_arrays[f"{name}/{key}"] = value.contiguous().to(torch.float32).numpy()
        block_manifest.append({"name": name, "config": {
            "dim": dim, "heads": heads, "kv_heads": kv_heads, "rope_theta": config.rope_theta, "layers": 12,
            "path_sdpa": config.path_sdpa, "sbda_fused": config.sbda_fused, "sbda_backward": config.sbda_backward,
            "attention_backend": backend, "path_topology": topology, "ff_mode": config.ff_mode,
            "ff_mult": config.ff_mult, "ff_hidden": ff_hidden, "ff_bias": ff_bias, "dropout": config.dropout},
            "layer_index": layer_index, "valid_mask": valid_mask is not None, "seam_reset": seam_reset is not None})
    block_arrays["manifest"] = np.frombuffer(json.dumps({"cases": block_manifest}).encode(), dtype=np.uint8)
    block_out = os.path.join(os.path.dirname(args.out), "block_golden.npz")
    np.savez_compressed(block_out, **block_arrays)
    print(f"wrote {block_out}: {len(block_manifest)} cases")
    path_out = os.path.join(os.path.dirname(args.out), "path_golden.npz")
    np.savez_compressed(path_out, **path_arrays)
    print(f"wrote {path_out}: {len(path_manifest)} cases")


if __name__ == "__main__":
    main()
