"""bloth_b200 - B200 (sm_100a) kernels for Bloth's fused RMSNorm + RoPE path.

Drop-in for the reference's names on this path (bloth/bloth/__init__.py:18-42
and kernels/__init__.py:7-8):

    rms_norm, BlothRMSNorm, fused_norm_qkv, BlothFusedNormQKV, rope_embedding,
    BlothRoPE, patch_model, FastModel, kernels.rms_norm, kernels.bloth_rms_norm,
    kernels.fused_norm_rope, kernels.rope_embedding

plus fused_qk_norm_rope / BlothQKNormRoPE (q and k per-head norm + RoPE in one
launch, cos/sin from positions in-register or from HF tables), apply_rope_qk /
apply_rotary_pos_emb (RoPE of q and k in one launch), the (1 + w) weighting of
Gemma-family norms (weight_offset), fused_add_rms_norm (residual add + RMSNorm
in one pass), and patch_model(..., patch_attention=True, patch_residual=True),
which routes HF Qwen3 / Llama / Mistral / Qwen2 layers through them. The compute runs in hand-written
CUDA behind the C ABI of include/bloth_b200.h; importing this package does not
touch the GPU, and every op raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

__version__ = "0.2.0"

from . import kernels  # noqa: F401
from .kernels import (  # noqa: F401
    apply_rope,
    apply_rope_qk,
    apply_rotary_pos_emb,
    fused_add_rms_norm,
    fused_norm_rope,
    fused_qk_norm_rope,
)
from .modules import (  # noqa: F401
    BlothFusedNormQKV,
    BlothQKNormRoPE,
    BlothRMSNorm,
    BlothRoPE,
    fused_norm_qkv,
    rms_norm,
    rope_inv_freq,
)
from .kernels.rope import rope_embedding  # noqa: F401
from .patch import FastModel, patch_model  # noqa: F401
from ._lib import BlothDeviceFault, device_fault, kernel_launch_count  # noqa: F401

__all__ = [
    "device_fault",
    "kernel_launch_count",
    "BlothDeviceFault",
    "kernels",
    "rms_norm",
    "BlothRMSNorm",
    "fused_norm_qkv",
    "BlothFusedNormQKV",
    "fused_add_rms_norm",
    "fused_norm_rope",
    "fused_qk_norm_rope",
    "BlothQKNormRoPE",
    "rope_embedding",
    "apply_rope",
    "apply_rope_qk",
    "apply_rotary_pos_emb",
    "BlothRoPE",
    "rope_inv_freq",
    "patch_model",
    "FastModel",
]
