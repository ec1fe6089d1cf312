"""Per-layer source schedules (exact causal offsets) of every path topology.

Restates ``BiAttn/topology.py:3-155``: the names of ``PATH_TOPOLOGIES`` in the
reference's order, and for each the offsets one layer reads.  Offset ``0`` is
the position itself; the others are exact distances to earlier positions.
Duplicates are dropped keeping the first occurrence, as the reference's
``_unique_offsets`` does (``topology.py:20-21``).

The kernels serve any one to four distinct offsets (the reference's fused
ops take two or four).  Topologies whose layers have more sources (``torus``,
``high4``, ``h8f``, ``h8g``, ``dinat_like``, ...) are listed so schedules can
be computed and compared, but the attention op rejects them with the
reference's ``ValueError``.
"""

from __future__ import annotations

from typing import Callable

# Same names and order as the reference (topology.py:3-10); "sbda" last.
PATH_TOPOLOGIES = (
    "binary", "local_jump", "mesh", "torus", "butterfly", "high4",
    "radix4", "radix8", "mixed_local_radix4", "longformer_local",
    "sparse_local_stride", "dinat_like", "longnet_like", "power_attention",
    "h0", "h1", "h2", "h3", "h4_greedy", "h5", "h6", "h7", "h8",
    "h8a", "h8b", "h8c", "h8d", "h8e", "h8f", "h8g", "sbda",
)


def _unique(offsets) -> tuple[int, ...]:
    out: list[int] = []
    for offset in offsets:
        if offset >= 0 and offset not in out:
            out.append(int(offset))
    return tuple(out)


def sbda_stage(layer: int) -> str:
    """``topology.py:13-17``: layers 1-2 are binary, later layers local diffusion."""
    if layer < 1:
        raise ValueError("layer must be positive")
    return "binary" if layer <= 2 else "local_diffusion"


def _staged(*near: int) -> Callable[[int, int, int], tuple[int, ...]]:
    """Binary (0, 2^(l-1)) for layers 1-2, then the near offsets plus 2^(l-1)."""
    return lambda layer, s, total: (0, s) if layer <= 2 else _unique((*near, s))


def _mixed_local_radix4(layer: int, s: int, total: int) -> tuple[int, ...]:
    # Binary strides for the first half of the stack, radix-4 lanes after it
    # (topology.py:146-155).
    split = max(1, total // 2)
    level = layer - 1
    if level < split:
        return (0, s)
    radix = (2 ** split) * (4 ** (level - split))
    return tuple(q * radix for q in range(4))


# Each rule maps (layer, stride = 2^(layer-1), total_layers) to the offsets.
_RULES: dict[str, Callable[[int, int, int], tuple[int, ...]]] = {
    "h0": lambda layer, s, total: (0, s),
    "binary": lambda layer, s, total: (0, s),
    "h1": lambda layer, s, total: _unique((0, 1, 2, s)),
    "local_jump": lambda layer, s, total: _unique((0, 1, 2, s)),
    "h2": lambda layer, s, total: _unique((0, s, 3 * s)),
    "h3": lambda layer, s, total: _unique((0, *range(s, 2 * s))),
    "h4_greedy": lambda layer, s, total: _unique((0, 3 ** (layer - 1), 2 * 3 ** (layer - 1))),
    "h5": lambda layer, s, total: (0, 1, 2) if layer == 1 else (0, 2 * s),
    "h6": lambda layer, s, total: _unique((0, s, 2 * s + 1)),
    "h7": lambda layer, s, total: (0, 1, 2) if layer <= 2 else (0, s),
    "h8": _staged(0, 1, 2),
    "sbda": _staged(0, 1, 2),
    "h8c": _staged(0, 1, 2),
    "h8a": _staged(0, 1),
    "h8b": _staged(0, 2),
    "h8f": _staged(0, 1, 2, 3),
    "h8g": _staged(0, 1, 2, 3, 4),
    "h8d": lambda layer, s, total: (0, 1, 2, s) if layer >= 3 and layer % 2 == 1 else (0, s),
    "h8e": lambda layer, s, total: _unique((0, 1, 2, s)) if layer > max(2, total - 2) else (0, s),
    "mesh": lambda layer, s, total: _unique((0, 1, s, s + 1)),
    "torus": lambda layer, s, total: _unique((0, 1, max(1, s - 1), s, s + 1)),
    "butterfly": lambda layer, s, total: _unique((0, s, 2 * s, 3 * s)),
    "high4": lambda layer, s, total: _unique((0, 1, 2, s, 2 * s, 3 * s)),
    "longformer_local": lambda layer, s, total: (0, 1, 2, 3),
    "sparse_local_stride": lambda layer, s, total: _unique((0, 1, 2, 3, max(4, 2 ** max(1, total // 2)))),
    "dinat_like": lambda layer, s, total: _unique((0, 1, 2, 3, 2 * s, 4 * s, 6 * s)),
    "longnet_like": lambda layer, s, total: _unique((0, 1, 2, 3, s, 2 * s, 3 * s)),
    "power_attention": lambda layer, s, total: _unique((0, 1, 2, 3, *(1 << e for e in range(total)))),
    "radix4": lambda layer, s, total: tuple(q * 4 ** (layer - 1) for q in range(4)),
    "radix8": lambda layer, s, total: tuple(q * 8 ** (layer - 1) for q in range(8)),
    "mixed_local_radix4": _mixed_local_radix4,
}


def topology_offsets(layer: int, *, topology: str = "binary", total_layers: int = 12) -> tuple[int, ...]:
    """Exact left offsets of one layer (``topology.py:24-155``).

    The default topology is ``"binary"``, as in the reference (``topology.py:24-28``); SBDA
    stacks pass ``topology="sbda"`` (or use :func:`sbda_layer_offsets`).
    """
    if layer < 1:
        raise ValueError("layer must be positive")
    if total_layers < 1:
        raise ValueError("total_layers must be positive")
    if topology not in PATH_TOPOLOGIES:
        raise ValueError(f"unknown path topology: {topology}")
    return _RULES[topology](layer, 2 ** (layer - 1), total_layers)


def sbda_layer_offsets(layers: int) -> list[tuple[int, ...]]:
    """Offsets of layers 1..layers of an SBDA stack."""
    return [topology_offsets(layer, topology="sbda", total_layers=layers) for layer in range(1, layers + 1)]
