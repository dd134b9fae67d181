"""Residual add + RMSNorm in one pass over the rows, with autograd.

``fused_add_rms_norm(x, residual, weight, eps=1e-6, weight_offset=0.0)``
returns ``(y, z)``: ``z = x + residual`` rounded to the input dtype (the new
residual stream) and ``y = RMSNorm(z) * (weight + weight_offset)``. It
replaces HF's ``hidden_states = residual + hidden_states`` followed by
``post_attention_layernorm(hidden_states)`` in Llama-family decoder layers
(transformers models/llama/modeling_llama.py, LlamaDecoderLayer.forward):
the rows are read once and written twice instead of read three times and
written twice by two kernels; the backward writes ``dz_out + dRMSNorm(dy)``
once, the gradient of both inputs. The reference has no residual fusion; the
RMSNorm part follows bloth/bloth/kernels/rms_norm.py:39-113.
"""
from __future__ import annotations

import torch

from .. import _lib
from .rms_norm import _as_rows, _check_row


class _AddRMSNormFunction(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, residual, weight, eps, weight_offset):
        _lib.require_cuda(x, residual, weight)
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("[Bloth] x and residual must have the same shape and dtype")
        shape = x.shape
        N = x.shape[-1]
        _check_row(N, x.dtype)
        x2, r2 = _as_rows(x, N), _as_rows(residual, N)
        M = x2.shape[0]
        y = torch.empty((M, N), dtype=x.dtype, device=x.device)
        z = torch.empty((M, N), dtype=x.dtype, device=x.device)
        rstd = torch.empty(M, dtype=torch.float32, device=x.device)
        rc = _lib.call("bloth_add_rmsnorm_fwd", x2, _lib.ptr(x2), x2.stride(0), _lib.ptr(r2),
                       r2.stride(0), _lib.ptr(z), z.stride(0), _lib.ptr(weight),
                       float(weight_offset), _lib.ptr(y), y.stride(0), _lib.ptr(rstd), M, N,
                       float(eps), _lib.dtype_code(x.dtype), _lib.dtype_code(weight.dtype),
                       _lib.stream_of(x2))
        _lib.check(rc, "add+rmsnorm forward")
        ctx.save_for_backward(z, weight, rstd)
        ctx.shape, ctx.weight_offset = shape, weight_offset
        return y.view(shape), z.view(shape)

    @staticmethod
    def backward(ctx, dy, dz_out):
        z, weight, rstd = ctx.saved_tensors
        M, N = z.shape
        dy2 = _as_rows(dy, N) if dy is not None else torch.zeros_like(z)
        dz2 = None if dz_out is None else _as_rows(dz_out, N)
        dz = torch.empty((M, N), dtype=z.dtype, device=z.device)
        dw = torch.empty(N, dtype=weight.dtype, device=z.device)
        ws_bytes = _lib.workspace_bytes("bloth_add_rmsnorm_bwd_workspace_bytes", z.device, M, N,
                                        _lib.dtype_code(z.dtype))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=z.device)
        rc = _lib.call("bloth_add_rmsnorm_bwd", z, _lib.ptr(dy2), dy2.stride(0), _lib.ptr(dz2),
                       dz2.stride(0) if dz2 is not None else N, _lib.ptr(z), z.stride(0),
                       _lib.ptr(weight), float(ctx.weight_offset), _lib.ptr(rstd), _lib.ptr(dz),
                       dz.stride(0), _lib.ptr(dw), M, N, _lib.dtype_code(z.dtype),
                       _lib.dtype_code(weight.dtype), _lib.ptr(ws), ws_bytes,
                       _lib.stream_of(z))
        _lib.check(rc, "add+rmsnorm backward")
        dz = dz.view(ctx.shape)
        return dz, dz, dw, None, None


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                       eps: float = 1e-6, weight_offset: float = 0.0):
    """(y, z): z = x + residual (in x's dtype), y = RMSNorm(z) * (weight +
    weight_offset) in fp32 rounded once. Gradients flow to x, residual and
    weight; z's gradient from later layers is added in the same kernel."""
    return _AddRMSNormFunction.apply(x, residual, weight.contiguous(), float(eps),
                                     float(weight_offset))
