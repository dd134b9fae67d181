"""Fused RMSNorm + rotate-half RoPE: autograd Functions over the sm_100a kernels.

Two entry points:

* ``fused_norm_rope(x, weight, cos, sin, eps=1e-6)`` - the reference's
  contract (bloth/bloth/kernels/fused_norm_qkv_rope.py:179-203): rows of N,
  per-row cos/sin tables [..., half] with numel M*half, columns >= 2*half
  normalised only. Same saved tensors and the same ``AssertionError`` on
  CPU tensors (:133). Its backward is the gradient of the forward (the
  reference's backward kernel :99-126 leaves out the transposed rotation).
* ``fused_qk_norm_rope(q, k, wq, wk, position_ids, inv_freq, eps)`` - q and
  k head tensors [B, S, H, D] normalised per head and rotated in one launch,
  cos/sin evaluated in-register from the positions (or read from tables),
  weight gradients for both.
"""
from __future__ import annotations

import torch

from .. import _lib
from .rms_norm import _as_rows, _check_row


# ---------------------------------------------------------------- row tables
def norm_rope_forward(x2, weight, cos2, sin2, eps, weight_offset=0.0):
    M, N = x2.shape
    half = cos2.shape[-1]
    y = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x2.device)
    rc = _lib.call("bloth_norm_rope_fwd", x2, _lib.ptr(x2), x2.stride(0), _lib.ptr(weight),
                   float(weight_offset), _lib.ptr(cos2), _lib.ptr(sin2), cos2.stride(0), _lib.dtype_code(cos2.dtype),
                   half, _lib.ptr(y), y.stride(0), _lib.ptr(rstd), M, N, float(eps),
                   _lib.dtype_code(x2.dtype), _lib.dtype_code(weight.dtype), _lib.stream_of(x2))
    _lib.check(rc, "fused norm+rope forward")
    return y, rstd


def norm_rope_backward(dy2, x2, weight, cos2, sin2, rstd, weight_offset=0.0):
    M, N = x2.shape
    half = cos2.shape[-1]
    dx = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    dw = torch.empty(N, dtype=weight.dtype, device=x2.device)
    ws_bytes = _lib.workspace_bytes("bloth_norm_rope_bwd_workspace_bytes", x2.device, M, N,
                                    _lib.dtype_code(x2.dtype))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x2.device)
    rc = _lib.call("bloth_norm_rope_bwd", x2, _lib.ptr(dy2), dy2.stride(0), _lib.ptr(x2),
                   x2.stride(0), _lib.ptr(weight), float(weight_offset), _lib.ptr(cos2),
                   _lib.ptr(sin2), cos2.stride(0),
                   _lib.dtype_code(cos2.dtype), half, _lib.ptr(rstd), _lib.ptr(dx), dx.stride(0),
                   _lib.ptr(dw), M, N, _lib.dtype_code(x2.dtype), _lib.dtype_code(weight.dtype),
                   _lib.ptr(ws), ws_bytes, _lib.stream_of(x2))
    _lib.check(rc, "fused norm+rope backward")
    return dx, dw


class _FusedNormRoPEFunction(torch.autograd.Function):
    """Reference: bloth/bloth/kernels/fused_norm_qkv_rope.py:129-176."""

    @staticmethod
    def forward(ctx, x, weight, cos, sin, eps=1e-6, weight_offset=0.0):
        assert x.is_cuda, "[Bloth] CUDA GPU required"
        _lib.require_cuda(weight, cos, sin)
        orig = x.shape
        N = x.shape[-1]
        _check_row(N, x.dtype)
        x2 = _as_rows(x, N)
        M = x2.shape[0]
        cos2 = _lib.aligned16(cos.contiguous().view(M, -1))
        sin2 = _lib.aligned16(sin.contiguous().view(M, -1))
        y, rstd = norm_rope_forward(x2, weight, cos2, sin2, eps, weight_offset)
        ctx.save_for_backward(x2, weight, rstd, cos2, sin2)
        ctx.eps = eps
        ctx.weight_offset = weight_offset
        ctx.orig = orig
        return y.view(orig)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd, cos2, sin2 = ctx.saved_tensors
        dy2 = _as_rows(dy, x2.shape[1])
        dx, dw = norm_rope_backward(dy2, x2, weight, cos2, sin2, rstd, ctx.weight_offset)
        return dx.view(ctx.orig), dw, None, None, None, None


def fused_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor,
                    sin: torch.Tensor, eps: float = 1e-6,
                    weight_offset: float = 0.0) -> torch.Tensor:
    """RMSNorm over the last dim of x, then rotate-half RoPE on its first
    2*cos.shape[-1] columns with per-row cos/sin. Same contract as
    bloth/bloth/kernels/fused_norm_qkv_rope.py:179-203; weight_offset (not in
    the reference) is added to the weight, 1.0 for Gemma-style norms."""
    return _FusedNormRoPEFunction.apply(x, weight.contiguous(), cos.contiguous(),
                                        sin.contiguous(), eps, float(weight_offset))


# ------------------------------------------------ per-head q/k (positions)
def _vec(dtype: torch.dtype) -> int:
    return 16 // torch.tensor([], dtype=dtype).element_size()


def _heads(t: torch.Tensor | None):
    """[B, S, H, D] view (3-D [S, H, D] gets B = 1) whose last dim is
    contiguous, 16-byte aligned and with strides the kernel can address."""
    if t is None:
        return None
    if t.dim() == 3:
        t = t.unsqueeze(0)
    if t.dim() != 4:
        raise ValueError("[Bloth] head tensors must be [B, S, H, D] or [S, H, D]")
    v = _vec(t.dtype)
    if (t.stride(3) != 1 or t.data_ptr() % 16 or any(s % v for s in t.stride()[:3])):
        t = _lib.aligned16(t.contiguous())
    return t


def _head_strides(t):
    return _lib.strides(t.stride()[:3]) if t is not None else None


def _positions(position_ids, B: int, S: int):
    """(tensor, strides[2]) for position ids of shape [S], [1, S] or [B, S]."""
    if position_ids is None:
        return None, None
    p = position_ids
    if p.dtype not in (torch.int32, torch.int64):
        p = p.long()
    if p.dim() == 1:
        p = p.unsqueeze(0)
    if p.shape[-1] != S or p.shape[0] not in (1, B):
        raise ValueError(f"[Bloth] position_ids shape {tuple(position_ids.shape)} does not "
                         f"match batch {B} x seq {S}")
    sb = 0 if p.shape[0] == 1 else p.stride(0)
    return p, _lib.strides((sb, p.stride(1)))


def _tables(cos, sin, B: int, S: int, D: int):
    """(cos, sin, strides[2], rows, token_indexed) for cos/sin tables.

    [P, D/2] or [P, D] tables are indexed by position; [B|1, S, D/2|D] tables
    (HuggingFace's position_embeddings) are indexed by token."""
    if cos is None and sin is None:
        return None, None, None, 0, False
    if cos is None or sin is None or cos.shape != sin.shape:
        raise ValueError("[Bloth] cos and sin must be given together with equal shapes")
    if cos.shape[-1] not in (D // 2, D):
        raise ValueError(f"[Bloth] cos/sin last dim must be {D // 2} or {D}")
    cos = _lib.aligned16(cos if cos.stride(-1) == 1 else cos.contiguous())
    sin = _lib.aligned16(sin if sin.stride(-1) == 1 else sin.contiguous())
    if cos.stride() != sin.stride():
        cos, sin = _lib.aligned16(cos.contiguous()), _lib.aligned16(sin.contiguous())
    if cos.dim() == 2:
        return cos, sin, _lib.strides((0, cos.stride(0))), cos.shape[0], False
    if cos.dim() == 3 and cos.shape[1] == S and cos.shape[0] in (1, B):
        sb = 0 if cos.shape[0] == 1 else cos.stride(0)
        return cos, sin, _lib.strides((sb, cos.stride(1))), S, True
    raise ValueError(f"[Bloth] unsupported cos/sin shape {tuple(cos.shape)}")


class _QKNormRoPEFunction(torch.autograd.Function):

    @staticmethod
    def forward(ctx, q, k, wq, wk, position_ids, inv_freq, cos, sin, eps, weight_offset,
                rope_scale):
        assert q.is_cuda, "[Bloth] CUDA GPU required"
        _lib.require_cuda(k, wq, wk, position_ids, inv_freq, cos, sin)
        shape_q = q.shape
        shape_k = None if k is None else k.shape
        q4, k4 = _heads(q), _heads(k)
        B, S, Hq, D = q4.shape
        Hk = 0 if k4 is None else k4.shape[2]
        if k4 is not None and (k4.shape[0] != B or k4.shape[1] != S or k4.shape[3] != D):
            raise ValueError("[Bloth] q and k must share batch, sequence and head_dim")
        pos, pos_st = _positions(position_ids, B, S)
        cos, sin, cs_st, cs_rows, token_idx = _tables(cos, sin, B, S, D)
        if (cos is None) == (inv_freq is None):
            raise ValueError("[Bloth] give exactly one of inv_freq or cos/sin")
        if inv_freq is not None:
            inv_freq = inv_freq.to(torch.float32).contiguous()
            if inv_freq.numel() != D // 2:
                raise ValueError(f"[Bloth] inv_freq must have head_dim/2 = {D // 2} elements")
        wq = _lib.aligned16(wq.contiguous())
        wk = None if wk is None else _lib.aligned16(wk.contiguous())
        if k4 is not None and wk is None:
            raise ValueError("[Bloth] wk is required with k")
        qo = torch.empty((B, S, Hq, D), dtype=q4.dtype, device=q4.device)
        ko = None if k4 is None else torch.empty((B, S, Hk, D), dtype=k4.dtype, device=k4.device)
        rq = torch.empty((B, S, Hq), dtype=torch.float32, device=q4.device)
        rk = None if k4 is None else torch.empty((B, S, Hk), dtype=torch.float32, device=q4.device)
        kpos = None if token_idx else pos
        rc = _lib.call(
            "bloth_qk_norm_rope_fwd", q4, _lib.ptr(q4), _head_strides(q4), _lib.ptr(k4),
            _head_strides(k4), _lib.ptr(wq), _lib.ptr(wk), float(weight_offset), _lib.ptr(qo),
            _head_strides(qo), _lib.ptr(ko), _head_strides(ko), _lib.ptr(rq), _lib.ptr(rk),
            _lib.ptr(kpos), pos_st if kpos is not None else None,
            _lib.dtype_code(kpos.dtype) if kpos is not None else 0, _lib.ptr(inv_freq),
            _lib.ptr(cos), _lib.ptr(sin), cs_st, cs_rows,
            _lib.dtype_code(cos.dtype) if cos is not None else 0, float(rope_scale), B, S, Hq,
            Hk, D, float(eps), _lib.dtype_code(q4.dtype), _lib.dtype_code(wq.dtype),
            _lib.stream_of(q4))
        _lib.check(rc, "qk norm+rope forward")
        ctx.save_for_backward(q4, k4, wq, wk, rq, rk, kpos, inv_freq, cos, sin)
        ctx.meta = (B, S, Hq, Hk, D, pos_st if kpos is not None else None, cs_st, cs_rows,
                    shape_q, shape_k, weight_offset, rope_scale)
        if k4 is None:
            return qo.view(shape_q)
        return qo.view(shape_q), ko.view(shape_k)

    @staticmethod
    def backward(ctx, *grads):
        q4, k4, wq, wk, rq, rk, pos, inv_freq, cos, sin = ctx.saved_tensors
        B, S, Hq, Hk, D, pos_st, cs_st, cs_rows, shape_q, shape_k, w_off, cs_scale = ctx.meta
        gq = _heads(grads[0].reshape(q4.shape) if grads[0].dim() != 4 else grads[0])
        gk = None
        if k4 is not None:
            g = grads[1]
            gk = _heads(g.reshape(k4.shape) if g.dim() != 4 else g)
        dq = torch.empty_like(q4, memory_format=torch.contiguous_format)
        dk = None if k4 is None else torch.empty_like(k4, memory_format=torch.contiguous_format)
        dwq = torch.empty(D, dtype=wq.dtype, device=q4.device)
        dwk = None if k4 is None else torch.empty(D, dtype=wk.dtype, device=q4.device)
        ws_bytes = _lib.workspace_bytes("bloth_qk_norm_rope_bwd_workspace_bytes", q4.device, B,
                                        S, D, _lib.dtype_code(q4.dtype))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q4.device)
        rc = _lib.call(
            "bloth_qk_norm_rope_bwd", q4, _lib.ptr(gq), _head_strides(gq), _lib.ptr(gk),
            _head_strides(gk), _lib.ptr(q4), _head_strides(q4), _lib.ptr(k4), _head_strides(k4),
            _lib.ptr(wq), _lib.ptr(wk), float(w_off), _lib.ptr(rq), _lib.ptr(rk), _lib.ptr(dq),
            _head_strides(dq), _lib.ptr(dk), _head_strides(dk), _lib.ptr(dwq), _lib.ptr(dwk),
            _lib.ptr(pos), pos_st, _lib.dtype_code(pos.dtype) if pos is not None else 0,
            _lib.ptr(inv_freq), _lib.ptr(cos), _lib.ptr(sin), cs_st, cs_rows,
            _lib.dtype_code(cos.dtype) if cos is not None else 0, float(cs_scale), B, S, Hq, Hk,
            D, _lib.dtype_code(q4.dtype), _lib.dtype_code(wq.dtype), _lib.ptr(ws), ws_bytes,
            _lib.stream_of(q4))
        _lib.check(rc, "qk norm+rope backward")
        return (dq.view(shape_q), None if dk is None else dk.view(shape_k), dwq, dwk, None, None,
                None, None, None, None, None)


def fused_qk_norm_rope(q: torch.Tensor, k: torch.Tensor | None, wq: torch.Tensor,
                       wk: torch.Tensor | None, position_ids: torch.Tensor | None = None,
                       inv_freq: torch.Tensor | None = None, eps: float = 1e-6,
                       cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                       weight_offset: float = 0.0, rope_scale: float = 1.0):
    """Per-head RMSNorm + rotate-half RoPE of q [B, S, Hq, D] and k [B, S, Hk, D].

    Each (token, head) row of D is normalised with wq (q) or wk (k) and
    rotated in pairs (d, d + D/2). cos/sin come from ``inv_freq`` [D/2]
    (angle = float32(position) * inv_freq, evaluated in-register) or from
    ``cos``/``sin`` tables ([P, D/2|D] indexed by position, or HF's
    [B, S, D] indexed by token). ``position_ids`` [B, S] / [1, S] / [S]
    default to 0..S-1. ``weight_offset`` is added to both weights (1.0 for
    Gemma-style ``(1 + w)`` norms); ``rope_scale`` multiplies cos and sin (HF's
    ``attention_scaling``; HF tables already include it, so pass 1.0 with
    them). Returns (q_out, k_out), or q_out alone when k is None. Shapes and
    dtypes of the outputs follow the inputs.
    """
    return _QKNormRoPEFunction.apply(q, k, wq, wk, position_ids, inv_freq, cos, sin, eps,
                                     float(weight_offset), float(rope_scale))
