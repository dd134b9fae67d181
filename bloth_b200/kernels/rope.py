"""Rotate-half RoPE alone, with autograd, over the sm_100a per-head kernel.

``rope_embedding(x, cos, sin, position_ids=None)`` keeps the reference's
signature and layout (bloth/bloth/ops/rope.py:33-58: x [b, h, s, d],
cos/sin [s, d/2]); ``apply_rope`` takes [B, S, H, D] tensors and either
inv_freq (cos/sin in-register) or tables; ``apply_rope_qk`` rotates q and k
in one launch; ``apply_rotary_pos_emb`` is a drop-in for the HuggingFace
function of that name (q, k [B, H, S, D], cos/sin [B, S, D]). Unlike the
reference, which is forward-only and always rounds to bf16 (:29-30), the
outputs keep the inputs' dtype and the backward (the transposed rotation)
is provided.
"""
from __future__ import annotations

import torch

from .. import _lib
from .fused_norm_qkv_rope import _head_strides, _heads, _positions, _tables


def _rope_launch(q4, qo, k4, ko, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows, scale: float,
                 transpose: bool):
    B, S, Hq, D = q4.shape
    Hk = 0 if k4 is None else k4.shape[2]
    rc = _lib.call("bloth_rope", q4, _lib.ptr(q4), _head_strides(q4), _lib.ptr(qo),
                   _head_strides(qo), _lib.ptr(k4), _head_strides(k4), _lib.ptr(ko),
                   _head_strides(ko), _lib.ptr(pos), pos_st,
                   _lib.dtype_code(pos.dtype) if pos is not None else 0, _lib.ptr(inv_freq),
                   _lib.ptr(cos), _lib.ptr(sin), cs_st, cs_rows,
                   _lib.dtype_code(cos.dtype) if cos is not None else 0, float(scale), B, S, Hq,
                   Hk, D, 1 if transpose else 0, _lib.dtype_code(q4.dtype), _lib.stream_of(q4))
    _lib.check(rc, "rope")


def _out_like(x4):
    """Output buffer with x4's strides when they are dense, else contiguous."""
    y = torch.empty_like(x4)
    if y.stride() != x4.stride():
        y = torch.empty(x4.shape, dtype=x4.dtype, device=x4.device)
    return y


class _RoPEFunction(torch.autograd.Function):
    """q4 [B, S, Hq, D] and optional k4 [B, S, Hk, D] views (any strides the
    kernel accepts); returns the rotated q, or (q, k)."""

    @staticmethod
    def forward(ctx, q4, k4, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows, scale):
        qo = _out_like(q4)
        ko = None if k4 is None else _out_like(k4)
        _rope_launch(q4, qo, k4, ko, pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows, scale,
                     False)
        ctx.save_for_backward(pos, inv_freq, cos, sin)
        ctx.cs_st, ctx.pos_st, ctx.cs_rows, ctx.scale = cs_st, pos_st, cs_rows, scale
        ctx.has_k = k4 is not None
        return qo if k4 is None else (qo, ko)

    @staticmethod
    def backward(ctx, *grads):
        pos, inv_freq, cos, sin = ctx.saved_tensors
        gq = _heads(grads[0])
        gk = _heads(grads[1]) if ctx.has_k else None
        dq = torch.empty(gq.shape, dtype=gq.dtype, device=gq.device)
        dk = None if gk is None else torch.empty(gk.shape, dtype=gk.dtype, device=gk.device)
        _rope_launch(gq, dq, gk, dk, pos, ctx.pos_st, inv_freq, cos, sin, ctx.cs_st, ctx.cs_rows,
                     ctx.scale, True)
        return dq, dk, None, None, None, None, None, None, None, None


def _rope_source(x4, position_ids, inv_freq, cos, sin):
    B, S, _, D = x4.shape
    pos, pos_st = _positions(position_ids, B, S)
    cos, sin, cs_st, cs_rows, token_idx = _tables(cos, sin, B, S, D)
    if (cos is None) == (inv_freq is None):
        raise ValueError("[Bloth] give exactly one of inv_freq or cos/sin")
    if inv_freq is not None:
        inv_freq = inv_freq.to(torch.float32).contiguous()
        if inv_freq.numel() != D // 2:
            raise ValueError(f"[Bloth] inv_freq must have head_dim/2 = {D // 2} elements")
    if token_idx:
        pos, pos_st = None, None
    return pos, pos_st, inv_freq, cos, sin, cs_st, cs_rows


def apply_rope(x: torch.Tensor, position_ids: torch.Tensor | None = None,
               inv_freq: torch.Tensor | None = None, cos: torch.Tensor | None = None,
               sin: torch.Tensor | None = None, rope_scale: float = 1.0) -> torch.Tensor:
    """Rotate-half RoPE of x [B, S, H, D] (or [S, H, D]); cos and sin are
    multiplied by ``rope_scale`` (HF's attention_scaling; 1.0 with HF tables,
    which include it)."""
    _lib.require_cuda(x, position_ids, inv_freq, cos, sin)
    shape = x.shape
    x4 = _heads(x)
    src = _rope_source(x4, position_ids, inv_freq, cos, sin)
    return _RoPEFunction.apply(x4, None, *src, float(rope_scale)).view(shape)


def apply_rope_qk(q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor | None = None,
                  inv_freq: torch.Tensor | None = None, cos: torch.Tensor | None = None,
                  sin: torch.Tensor | None = None, rope_scale: float = 1.0):
    """Rotate-half RoPE of q [B, S, Hq, D] and k [B, S, Hk, D] in one launch,
    with the cos/sin rules of :func:`apply_rope`. Returns (q_out, k_out)."""
    _lib.require_cuda(q, k, position_ids, inv_freq, cos, sin)
    sq, sk = q.shape, k.shape
    q4, k4 = _heads(q), _heads(k)
    if k4.shape[0] != q4.shape[0] or k4.shape[1] != q4.shape[1] or k4.shape[3] != q4.shape[3]:
        raise ValueError("[Bloth] q and k must share batch, sequence and head_dim")
    src = _rope_source(q4, position_ids, inv_freq, cos, sin)
    qo, ko = _RoPEFunction.apply(q4, k4, *src, float(rope_scale))
    return qo.view(sq), ko.view(sk)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor, position_ids=None, unsqueeze_dim: int = 1):
    """Drop-in for HuggingFace's ``apply_rotary_pos_emb`` (transformers
    models/llama/modeling_llama.py): q [B, Hq, S, D], k [B, Hk, S, D],
    cos/sin [B, S, D] (the rotary embedding's output, attention scaling
    included). Both tensors rotate in one launch; the outputs are
    [B, H, S, D] views of [B, S, H, D] buffers."""
    if unsqueeze_dim != 1:
        raise ValueError("[Bloth] apply_rotary_pos_emb supports the [B, H, S, D] layout only")
    qo, ko = apply_rope_qk(q.transpose(1, 2), k.transpose(1, 2), cos=cos, sin=sin)
    return qo.transpose(1, 2), ko.transpose(1, 2)


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
