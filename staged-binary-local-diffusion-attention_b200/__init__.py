"""SBDA sparse gather-softmax attention for NVIDIA B200 (sm_100a).

Import as ``sbda_b200`` (the repository root's ``sbda_b200.py`` maps that
name onto this directory).  The compute runs in ``libsbda_b200.so`` (built
from ``csrc/`` by ``build.py``) behind the C ABI of ``include/sbda_b200.h``.
"""

from .ops import (
    current_family,
    device_status,
    fused_sbda,
    fused_sbda_block,
    fused_sbda_block_full,
    fused_sbda_gqa_key_backward,
    fused_sbda_key_backward,
    host_offsets,
    kernel_family,
    sbda_attention,
    sbda_backward,
    sbda_forward,
)
from .norm_rope import norm_rope, normed_attention, normed_supported, rope_table
from .topology import PATH_TOPOLOGIES, sbda_layer_offsets, sbda_stage, topology_offsets

__all__ = [
    "BiAttnBlock", "BiAttnConfig", "BiAttnLM", "BinaryPathAttention", "PATH_TOPOLOGIES", "RMSNorm", "SBDAttention", "SwiGLU",
    "add_rms_norm", "rms_norm", "silu_mul", "SBDAAttention", "current_family", "device_status", "kernel_family", "fused_sbda",
    "fused_sbda_block", "fused_sbda_block_full", "fused_sbda_gqa_key_backward",
    "fused_sbda_key_backward", "host_offsets", "norm_rope", "normed_attention", "normed_supported", "rope_table", "sbda_attention", "sbda_backward", "sbda_forward",
    "sbda_layer_offsets", "sbda_stage", "topology_offsets",
]


def __getattr__(name: str):
    if name in ("SBDAttention", "SBDAAttention", "BinaryPathAttention"):
        from . import attention

        return getattr(attention, name)
    if name in ("BiAttnConfig", "BiAttnLM", "FactorizedTokenIO"):
        from . import model

        return getattr(model, name)
    if name in ("BiAttnBlock", "RMSNorm", "SwiGLU", "add_rms_norm", "rms_norm", "silu_mul"):
        from . import block

        return getattr(block, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
