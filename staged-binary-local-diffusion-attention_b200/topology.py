"""Per-layer source schedules served by the SBDA kernels.

Restates ``BiAttn/topology.py`` for the topologies whose layers have at most
four sources with at most one beyond the kernel's near window: ``sbda``
(``topology.py:141-142``) and its relatives.  Offsets are exact causal
distances; ``0`` (self) comes first, duplicates are dropped in order
(``topology.py:20-21``).
"""

from __future__ import annotations

PATH_TOPOLOGIES = (
    "sbda", "h8", "h8a", "h8b", "h8c", "h8d", "h8e", "binary", "h0", "h1", "h7",
    "local_jump", "longformer_local",
)


def _unique(offsets: tuple[int, ...]) -> tuple[int, ...]:
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


def topology_offsets(layer: int, *, topology: str = "sbda", total_layers: int = 12) -> tuple[int, ...]:
    """Exact left offsets of one layer (``topology.py:24-155``, subset)."""
    if layer < 1:
        raise ValueError("layer must be positive")
    if total_layers < 1:
        raise ValueError("total_layers must be positive")
    if topology not in PATH_TOPOLOGIES:
        raise ValueError(f"unknown path topology: {topology}")
    stride = 2 ** (layer - 1)
    if topology in ("sbda", "h8", "h8c"):
        return (0, stride) if layer <= 2 else _unique((0, 1, 2, stride))
    if topology == "h8a":
        return (0, stride) if layer <= 2 else _unique((0, 1, stride))
    if topology == "h8b":
        return (0, stride) if layer <= 2 else _unique((0, 2, stride))
    if topology == "h8d":
        return (0, 1, 2, stride) if layer >= 3 and layer % 2 == 1 else (0, stride)
    if topology == "h8e":
        return _unique((0, 1, 2, stride)) if layer > max(2, total_layers - 2) else (0, stride)
    if topology in ("binary", "h0"):
        return (0, stride)
    if topology in ("h1", "local_jump"):
        return _unique((0, 1, 2, stride))
    if topology == "h7":
        return (0, 1, 2) if layer <= 2 else (0, stride)
    return (0, 1, 2, 3)  # longformer_local


def sbda_layer_offsets(layers: int) -> list[tuple[int, ...]]:
    """Offsets of layers 1..layers of an SBDA stack."""
    return [topology_offsets(layer, topology="sbda", total_layers=layers) for layer in range(1, layers + 1)]
