"""nn.Module wrappers with the reference's names and constructor arguments.

* ``BlothRMSNorm(hidden_size, eps=1e-6)`` - bloth/bloth/ops/rms_norm.py:7-19
* ``BlothFusedNormQKV(hidden_size, eps=1e-6).forward(x, cos, sin)`` -
  bloth/bloth/ops/fused_norm_qkv.py:7-28
* ``BlothRoPE(head_dim, max_seq_len=8192, base=10000.0)`` -
  bloth/bloth/ops/rope.py:61-82 (bf16 cos/sin caches, as the reference)
* ``BlothQKNormRoPE(head_dim, eps=1e-6, base=10000.0)`` - per-head q/k norm +
  RoPE with cos/sin evaluated in-register (no reference counterpart)
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .kernels.fused_norm_qkv_rope import fused_norm_rope, fused_qk_norm_rope
from .kernels.rms_norm import rms_norm as _rms_norm_fn
from .kernels.rope import rope_embedding


def rope_inv_freq(head_dim: int, base: float = 10000.0) -> torch.Tensor:
    """inv_freq [head_dim/2] fp32: 1/(base ** (arange(0, h)/h)), as
    BlothRoPE._build_cache (bloth/bloth/ops/rope.py:71)."""
    half = head_dim // 2
    return 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))


class BlothRMSNorm(nn.Module):
    """Drop-in for LlamaRMSNorm / MistralRMSNorm / Qwen*RMSNorm.

    ``weight_offset=1.0`` makes it a drop-in for GemmaRMSNorm, whose output is
    x_hat * (1 + weight) with weight initialised to zeros; the weight is then
    initialised to 1 - weight_offset so that a fresh module is the identity
    scale either way."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, weight_offset: float = 0.0):
        super().__init__()
        self.weight = nn.Parameter(torch.full((hidden_size,), 1.0 - weight_offset))
        self.eps = eps
        self.weight_offset = float(weight_offset)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _rms_norm_fn(x, self.weight, self.eps, self.weight_offset)

    def extra_repr(self) -> str:
        extra = f", weight_offset={self.weight_offset}" if self.weight_offset else ""
        return f"hidden_size={self.weight.shape[0]}, eps={self.eps}{extra}"


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             weight_offset: float = 0.0) -> torch.Tensor:
    return _rms_norm_fn(x, weight, eps, weight_offset)


class BlothFusedNormQKV(nn.Module):
    """RMSNorm + RoPE in one kernel over rows of ``hidden_size``, with per-row
    cos/sin [..., half] (reference: bloth/bloth/ops/fused_norm_qkv.py:7-28)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x, cos, sin):
        orig = x.shape
        N = x.shape[-1]
        M = x.numel() // N
        out = fused_norm_rope(x.reshape(M, N), self.weight, cos.reshape(M, -1),
                              sin.reshape(M, -1), self.eps)
        return out.view(orig)


def fused_norm_qkv(x, weight, cos, sin, eps=1e-6):
    return fused_norm_rope(x, weight, cos, sin, eps)


class BlothRoPE(nn.Module):
    """Pre-computes bf16 cos/sin caches [max_seq_len, head_dim/2]
    (reference: bloth/bloth/ops/rope.py:61-82)."""

    def __init__(self, head_dim: int, max_seq_len: int = 8192, base: float = 10000.0):
        super().__init__()
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.base = base
        self._build_cache(max_seq_len)

    def _build_cache(self, seq_len: int):
        inv_freq = rope_inv_freq(self.head_dim, self.base)
        t = torch.arange(seq_len, dtype=torch.float32)
        freqs = torch.outer(t, inv_freq)
        dev = getattr(self, "cos_cache", None)
        dev = dev.device if dev is not None else None
        self.register_buffer("cos_cache", freqs.cos().bfloat16().to(dev), persistent=False)
        self.register_buffer("sin_cache", freqs.sin().bfloat16().to(dev), persistent=False)
        self.max_seq_len = seq_len

    def forward(self, x: torch.Tensor, seq_len: int = None) -> torch.Tensor:
        need = seq_len or x.shape[2]
        if need > self.max_seq_len:
            self._build_cache(need)
        return rope_embedding(x, self.cos_cache, self.sin_cache)


class BlothQKNormRoPE(nn.Module):
    """q_norm / k_norm weights [head_dim] with fused per-head RMSNorm + RoPE of
    q [B, S, Hq, D] and k [B, S, Hk, D]; cos/sin from positions in-register."""

    def __init__(self, head_dim: int, eps: float = 1e-6, base: float = 10000.0):
        super().__init__()
        self.q_weight = nn.Parameter(torch.ones(head_dim))
        self.k_weight = nn.Parameter(torch.ones(head_dim))
        self.eps = eps
        self.register_buffer("inv_freq", rope_inv_freq(head_dim, base), persistent=False)

    def forward(self, q, k, position_ids=None):
        return fused_qk_norm_rope(q, k, self.q_weight, self.k_weight, position_ids,
                                  self.inv_freq, self.eps)
