"""RMSNorm autograd Function and functional op over the sm_100a kernels.

Mirrors the reference's bloth/bloth/kernels/rms_norm.py: same names
(``_RMSNormFunction``, ``rms_norm``, ``bloth_rms_norm``), same argument
meaning ``(x, weight, eps=1e-6)``, same saved tensors ``(x_2d, weight,
rstd_fp32[M])`` and the same size-limit error; the kernels behind it are the
C ABI's ``bloth_rmsnorm_fwd`` / ``bloth_rmsnorm_bwd``.
"""
from __future__ import annotations

import torch

from .. import _lib

MAX_FUSED_SIZE = 65536  # reference limit, bloth/bloth/kernels/rms_norm.py:21


def _max_row(dtype: torch.dtype) -> int:
    return 32768 if dtype == torch.float32 else MAX_FUSED_SIZE


def _check_row(n: int, dtype: torch.dtype) -> None:
    """RuntimeError for over-long rows, as bloth/bloth/kernels/rms_norm.py:27-31."""
    limit = _max_row(dtype)
    if n > limit:
        raise RuntimeError(
            f"[Bloth] RMSNorm: hidden_dim={n} exceeds max CUDA blocksize {limit}. "
            "Split your hidden dimension.")


def _as_rows(t: torch.Tensor, n: int) -> torch.Tensor:
    """2-D [M, n] view with unit column stride (copying only when needed)."""
    if t.dim() == 2 and t.stride(1) == 1 and (t.shape[0] <= 1 or t.stride(0) >= n):
        return _lib.aligned16(t) if t.data_ptr() % 16 else t
    return _lib.aligned16(t.contiguous().view(-1, n))


def rmsnorm_forward(x2: torch.Tensor, weight: torch.Tensor, eps: float,
                    weight_offset: float = 0.0):
    """y [M, N] (x's dtype) and rstd [M] fp32 for rows x2 [M, N]; the weight
    applied is weight + weight_offset (1.0 for Gemma-style norms)."""
    _lib.require_cuda(x2, weight)
    M, N = x2.shape
    _check_row(N, x2.dtype)
    y = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x2.device)
    rc = _lib.call("bloth_rmsnorm_fwd", x2, _lib.ptr(x2), x2.stride(0), _lib.ptr(weight),
                   float(weight_offset), _lib.ptr(y), y.stride(0), _lib.ptr(rstd), M, N, float(eps),
                   _lib.dtype_code(x2.dtype), _lib.dtype_code(weight.dtype), _lib.stream_of(x2))
    _lib.check(rc, "rmsnorm forward")
    return y, rstd


def rmsnorm_backward(dy2: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor,
                     rstd: torch.Tensor, weight_offset: float = 0.0):
    """dx [M, N] (x's dtype) and dweight [N] (weight's dtype)."""
    M, N = x2.shape
    dx = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    dw = torch.empty(N, dtype=weight.dtype, device=x2.device)
    ws_bytes = _lib.workspace_bytes("bloth_rmsnorm_bwd_workspace_bytes", x2.device, M, N,
                                    _lib.dtype_code(x2.dtype))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x2.device)
    rc = _lib.call("bloth_rmsnorm_bwd", x2, _lib.ptr(dy2), dy2.stride(0), _lib.ptr(x2),
                   x2.stride(0), _lib.ptr(weight), float(weight_offset), _lib.ptr(rstd), _lib.ptr(dx), dx.stride(0),
                   _lib.ptr(dw), M, N, _lib.dtype_code(x2.dtype), _lib.dtype_code(weight.dtype),
                   _lib.ptr(ws), ws_bytes, _lib.stream_of(x2))
    _lib.check(rc, "rmsnorm backward")
    return dx, dw


class _RMSNormFunction(torch.autograd.Function):
    """Reference: bloth/bloth/kernels/rms_norm.py:116-160."""

    @staticmethod
    def forward(ctx, x, weight, eps=1e-6, weight_offset=0.0):
        _lib.require_cuda(x, weight)
        orig_shape = x.shape
        N = x.shape[-1]
        _check_row(N, x.dtype)
        x2 = _as_rows(x, N)
        y, rstd = rmsnorm_forward(x2, weight, eps, weight_offset)
        ctx.save_for_backward(x2, weight, rstd)
        ctx.eps = eps
        ctx.weight_offset = weight_offset
        ctx.orig_shape = orig_shape
        return y.view(orig_shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        M, N = x2.shape
        dy2 = _as_rows(dy, N)
        dx, dw = rmsnorm_backward(dy2, x2, weight, rstd, ctx.weight_offset)
        return dx.view(ctx.orig_shape), dw, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             weight_offset: float = 0.0) -> torch.Tensor:
    """RMSNorm over the last dimension; drop-in for LlamaRMSNorm-style norms.

    Reference: bloth/bloth/kernels/rms_norm.py:163-176. y = x * rsqrt(mean(x^2)
    + eps) * (weight + weight_offset) in fp32, rounded once to x's dtype.
    weight_offset=1.0 gives the (1 + w) weighting of Gemma-family norms
    (transformers GemmaRMSNorm.forward); the reference has no such option.
    """
    return _RMSNormFunction.apply(x, weight.contiguous(), eps, float(weight_offset))


# the reference exports this alias (bloth/bloth/kernels/rms_norm.py:181)
bloth_rms_norm = rms_norm
