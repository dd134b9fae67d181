"""Rotate-half RoPE alone, with autograd, over the sm_100a per-head kernel.

``rope_embedding(x, cos, sin, position_ids=None)`` keeps the reference's
signature and layout (bloth/bloth/ops/rope.py:33-58: x [b, h, s, d],
cos/sin [s, d/2]); ``apply_rope`` takes [B, S, H, D] tensors and either
inv_freq (cos/sin in-register) or tables. Unlike the reference, which is
forward-only and always rounds to bf16 (:29-30), the output keeps x's dtype
and the backward (the transposed rotation) is provided.
"""
from __future__ import annotations

import torch

from .. import _lib
from .fused_norm_qkv_rope import _head_strides, _heads, _positions, _tables


def _rope_launch(x4, y4, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows, transpose: bool):
    B, S, H, D = x4.shape
    rc = _lib.call("bloth_rope", x4, _lib.ptr(x4), _head_strides(x4), _lib.ptr(y4),
                   _head_strides(y4), _lib.ptr(pos), pos_st,
                   _lib.dtype_code(pos.dtype) if pos is not None else 0, _lib.ptr(inv_freq),
                   _lib.ptr(cos), _lib.ptr(sin), cs_st, cs_rows,
                   _lib.dtype_code(cos.dtype) if cos is not None else 0, B, S, H, D,
                   1 if transpose else 0, _lib.dtype_code(x4.dtype), _lib.stream_of(x4))
    _lib.check(rc, "rope")


class _RoPEFunction(torch.autograd.Function):
    """x4: [B, S, H, D] view (any strides the kernel accepts)."""

    @staticmethod
    def forward(ctx, x4, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows):
        y4 = torch.empty_like(x4)
        if y4.stride() != x4.stride():
            y4 = torch.empty(x4.shape, dtype=x4.dtype, device=x4.device)
        _rope_launch(x4, y4, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows, False)
        ctx.save_for_backward(pos, inv_freq, cos, sin)
        ctx.cs_st, ctx.pos_st, ctx.cs_rows = cs_st, pos_st, cs_rows
        return y4

    @staticmethod
    def backward(ctx, dy4):
        pos, inv_freq, cos, sin = ctx.saved_tensors
        dy4 = _heads(dy4)
        dx4 = torch.empty(dy4.shape, dtype=dy4.dtype, device=dy4.device)
        _rope_launch(dy4, dx4, pos, ctx.pos_st, inv_freq, cos, sin, ctx.cs_st, ctx.cs_rows, True)
        return dx4, None, None, None, None, None, None, None


def apply_rope(x: torch.Tensor, position_ids: torch.Tensor | None = None,
               inv_freq: torch.Tensor | None = None, cos: torch.Tensor | None = None,
               sin: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate-half RoPE of x [B, S, H, D] (or [S, H, D])."""
    _lib.require_cuda(x, position_ids, inv_freq, cos, sin)
    shape = x.shape
    x4 = _heads(x)
    B, S, H, D = x4.shape
    pos, pos_st = _positions(position_ids, B, S)
    cos, sin, cs_st, cs_rows, token_idx = _tables(cos, sin, B, S, D)
    if (cos is None) == (inv_freq is None):
        raise ValueError("[Bloth] give exactly one of inv_freq or cos/sin")
    if inv_freq is not None:
        inv_freq = inv_freq.to(torch.float32).contiguous()
    if token_idx:
        pos, pos_st = None, None
    return _RoPEFunction.apply(x4, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows).view(shape)


def rope_embedding(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   position_ids: torch.Tensor | None = None) -> torch.Tensor:
    """Rotary embedding of x [batch, heads, seq, head_dim] with cos/sin
    [seq_or_positions, head_dim/2]; row p of the tables serves position p
    (``position_ids`` [batch, seq] if given, else the sequence index).
    Reference: bloth/bloth/ops/rope.py:33-58."""
    _lib.require_cuda(x, cos, sin, position_ids)
    # [b, h, s, d] seen as tokens (b, s) with heads h: swap the middle axes
    # of the view only; no data moves.
    x4 = _heads(x.transpose(1, 2))
    out = apply_rope(x4, position_ids=position_ids, cos=cos, sin=sin)
    return out.transpose(1, 2)
