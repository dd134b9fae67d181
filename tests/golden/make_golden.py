"""Generates the golden vectors in this folder from the reference itself.

Runs shell-bay/bloth's own Triton kernels on the CPU through Triton's
interpreter (TRITON_INTERPRET=1) and stores their inputs and outputs as
compressed .npz files. Only needs the reference checkout, which exists in the
build container (not on GPU machines); the committed .npz files are what the
tests read.

    python tests/golden/make_golden.py /path/to/reference/bloth
    (or BLOTH_REFERENCE=/path/to/reference/bloth python tests/golden/make_golden.py)

Vectors written (all seeded):
  rmsnorm_f32.npz      reference rms_norm fwd (y, rstd) and bwd (dx, dw), fp32
  rmsnorm_bf16.npz     reference rms_norm fwd, bf16 x with unit weight, the
                       reference test's own golden case shape (M=256, N=2048)
  fused_q_f32.npz      fused_norm_rope fwd kernel, the q tensor of the CPU
                       correctness config (q [2,128,8,64], theta 1e4)
  fused_k_f32.npz      same for k [2,128,2,64], plus the reference bwd kernel
  fused_rest_bf16.npz  fused kernel on rows wider than the rotated part
                       (N=256, half=32), bf16, plus the reference bwd kernel
  rope_bf16.npz        rope_embedding forward (bf16 store), x [2,4,16,64]
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BLOTH_REFERENCE")


def f32(t: torch.Tensor) -> np.ndarray:
    """fp32 tensors as float32 arrays; bf16 tensors as their uint16 bit patterns
    (tests/golden/__init__.py:load turns uint16 arrays back into bf16)."""
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.to(torch.float32).numpy()


def normal(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def weight(n, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(n, generator=g)).to(dtype)


def main() -> None:
    if not REF or not os.path.isdir(os.path.join(REF, "bloth")):
        raise SystemExit("make_golden.py: give the reference checkout's bloth/ directory as "
                         "the first argument or in BLOTH_REFERENCE")
    sys.path.insert(0, REF)
    from bloth.kernels.rms_norm import rms_norm, _rms_norm_fwd_kernel, _calculate_settings
    from bloth.kernels.fused_norm_qkv_rope import (
        _fused_norm_rope_fwd_kernel,
        _fused_norm_rope_bwd_kernel,
        _calculate_settings as _fused_settings,
    )
    from bloth.ops.rope import rope_embedding, BlothRoPE

    # --- rms_norm fp32 fwd + bwd through the reference autograd Function
    M, N, eps = 64, 256, 1e-6
    x = normal((M, N), 1).requires_grad_(True)
    w = weight(N, 2).requires_grad_(True)
    dy = normal((M, N), 3)
    y = rms_norm(x, w, eps)
    y.backward(dy)
    rstd = torch.empty(M)
    bs, nw = _calculate_settings(N)
    _rms_norm_fwd_kernel[(M,)](torch.empty(M, N), x.detach(), w.detach(), rstd, N, N, N, eps,
                               BLOCK_SIZE=bs, num_warps=nw)
    np.savez_compressed(os.path.join(HERE, "rmsnorm_f32.npz"), x=f32(x), w=f32(w), dy=f32(dy),
                        y=f32(y), rstd=f32(rstd), dx=f32(x.grad), dw=f32(w.grad), eps=eps)

    # --- rms_norm bf16 forward, the reference test's shape (test_kernels.py:119-121)
    M, N = 256, 2048
    xb = normal((M, N), 4, torch.bfloat16)
    wb = torch.ones(N, dtype=torch.bfloat16)
    yb = rms_norm(xb, wb)
    np.savez_compressed(os.path.join(HERE, "rmsnorm_bf16.npz"), x=f32(xb), w=f32(wb), y=f32(yb),
                        eps=1e-6)

    # --- fused norm+rope, CPU correctness config: q [2,128,8,64], k [2,128,2,64]
    theta, eps, D, S = 1e4, 1e-6, 64, 128
    half = D // 2
    inv_f = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    freqs = torch.outer(torch.arange(S, dtype=torch.float32), inv_f)
    cos_t, sin_t = freqs.cos(), freqs.sin()  # fp32 tables [S, half]

    def fused_fwd(x2, w_, cos_rows, sin_rows, eps_):
        Mx, Nx = x2.shape
        yy = torch.empty_like(x2)
        rs = torch.empty(Mx, dtype=torch.float32)
        bs_, nw_ = _fused_settings(Nx)
        _fused_norm_rope_fwd_kernel[(Mx,)](yy, x2, w_, rs, cos_rows, sin_rows, x2.stride(0),
                                           yy.stride(0), cos_rows.stride(0), Nx, eps_,
                                           cos_rows.shape[-1], BLOCK_SIZE=bs_, num_warps=nw_)
        return yy, rs

    def fused_bwd(dy2, x2, w_, rs):
        Mx, Nx = x2.shape
        dx = torch.empty_like(x2)
        dw = torch.zeros(Nx, dtype=torch.float32)
        bs_, nw_ = _fused_settings(Nx)
        _fused_norm_rope_bwd_kernel[(Mx,)](dx, dw, dy2, x2, w_, rs, x2.stride(0), dy2.stride(0),
                                           Nx, BLOCK_SIZE=bs_, num_warps=nw_)
        return dx, dw

    for name, H, seed in (("q", 8, 10), ("k", 2, 20)):
        xt = normal((2, S, H, D), seed)
        wt = weight(D, seed + 1)
        pos = torch.arange(S).view(1, S, 1).expand(2, S, H).reshape(-1)
        cos_rows = cos_t[pos].contiguous()
        sin_rows = sin_t[pos].contiguous()
        x2 = xt.view(-1, D)
        yt, rs = fused_fwd(x2, wt, cos_rows, sin_rows, eps)
        out = dict(x=f32(xt), w=f32(wt), cos=f32(cos_t), sin=f32(sin_t), y=f32(yt.view_as(xt)),
                   rstd=f32(rs), theta=theta, eps=eps)
        if name == "k":
            dyt = normal((2, S, H, D), seed + 2)
            dx, dw = fused_bwd(dyt.view(-1, D), x2, wt, rs)
            out.update(dy=f32(dyt), ref_bwd_dx=f32(dx.view_as(xt)), ref_bwd_dw=f32(dw))
        np.savez_compressed(os.path.join(HERE, f"fused_{name}_f32.npz"), **out)

    # --- fused kernel on rows wider than the rotated part, bf16
    M, N, h = 48, 256, 32
    xr = normal((M, N), 30, torch.bfloat16)
    wr = weight(N, 31, torch.bfloat16)
    cr = normal((M, h), 32).clamp(-1, 1)
    sr = torch.sqrt(1 - cr * cr)
    yr, rsr = fused_fwd(xr, wr, cr, sr, 1e-5)
    dyr = normal((M, N), 33, torch.bfloat16)
    dxr, dwr = fused_bwd(dyr, xr, wr, rsr)
    np.savez_compressed(os.path.join(HERE, "fused_rest_bf16.npz"), x=f32(xr), w=f32(wr),
                        cos=f32(cr), sin=f32(sr), y=f32(yr), rstd=f32(rsr), dy=f32(dyr),
                        ref_bwd_dx=f32(dxr), ref_bwd_dw=f32(dwr), eps=1e-5)

    # --- rope_embedding forward with the BlothRoPE bf16 cache
    b, hh, s, d = 2, 4, 16, 64
    xe = normal((b, hh, s, d), 40, torch.bfloat16)
    mod = BlothRoPE(d, max_seq_len=s, base=1e4)
    ye = rope_embedding(xe, mod.cos_cache, mod.sin_cache)
    np.savez_compressed(os.path.join(HERE, "rope_bf16.npz"), x=f32(xe), cos=f32(mod.cos_cache),
                        sin=f32(mod.sin_cache), y=f32(ye), base=1e4)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
