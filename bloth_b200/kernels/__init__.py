"""Autograd Functions and functional ops over the sm_100a kernels.

Same names as the reference's ``bloth.kernels`` package for this path
(bloth/bloth/kernels/__init__.py:7-8): ``rms_norm``, ``bloth_rms_norm``,
``fused_norm_rope``; plus ``fused_qk_norm_rope``, ``fused_add_rms_norm`` and
the RoPE-only ops.
"""
from .rms_norm import bloth_rms_norm, rms_norm  # noqa: F401
from .add_rms_norm import fused_add_rms_norm  # noqa: F401
from .fused_norm_qkv_rope import fused_norm_rope, fused_qk_norm_rope  # noqa: F401
from .rope import apply_rope, apply_rope_qk, apply_rotary_pos_emb, rope_embedding  # noqa: F401

__all__ = [
    "bloth_rms_norm",
    "rms_norm",
    "fused_add_rms_norm",
    "fused_norm_rope",
    "fused_qk_norm_rope",
    "apply_rope",
    "apply_rope_qk",
    "apply_rotary_pos_emb",
    "rope_embedding",
]
