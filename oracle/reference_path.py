"""CPU restatement of the reference's RMSNorm / fused RMSNorm+RoPE math.

Test infrastructure: imported only by ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg, as the checker. Every forward below is a
plain PyTorch expression evaluated in ``compute`` precision (float64 by
default for parity checks; float32 reproduces the reference golden's own
precision for the CPU timing baseline). Backward passes are
``torch.autograd`` of those forwards, i.e. the exact gradient of the path.

Reference semantics restated (paths relative to the reference project):

* RMSNorm: ``x32 = x.float(); rms = sqrt(mean(x32**2) + eps);
  (x32 / rms * w.float()).to(dtype)`` - bloth/tests/test_kernels.py:124-127,
  the same math as the kernel bloth/bloth/kernels/rms_norm.py:59-73
  (``mean_sq = sum(x*x)/n; rstd = rsqrt(mean_sq + eps); y = x*rstd*w``).
* Fused norm + RoPE: the row is normalised over all N columns, then pairs
  (c, c+h) for c < h = cos.shape[-1] are rotated, ``y1 = x1*cos - x2*sin``,
  ``y2 = x1*sin + x2*cos``, columns >= 2h stay normalised only -
  bloth/bloth/kernels/fused_norm_qkv_rope.py:59-96. cos/sin are per row
  ([M, h], :138-141).
* cos/sin construction: ``inv_freq = 1/(base ** (arange(0, h)/h))``,
  ``freqs = outer(t, inv_freq)`` in float32, ``cos = freqs.cos()`` -
  bloth/bloth/ops/rope.py:71-75. The angle is rounded to float32 exactly as
  ``torch.outer`` does; only cos/sin of that float32 angle are evaluated in
  ``compute`` precision.
* RoPE alone: bloth/bloth/ops/rope.py:21-27 (same rotation, no norm).

Two extensions the reference does not have, restated from the third-party
code they serve (transformers 5.5.0 as installed):

* ``w_offset``: the weight enters as ``w + w_offset``; 1.0 is GemmaRMSNorm's
  ``_norm(x.float()) * (1.0 + weight.float())`` (models/gemma/
  modeling_gemma.py, GemmaRMSNorm.forward). The reference's patcher puts an
  ``x_hat * w`` norm in place of GemmaRMSNorm (bloth/bloth/patch.py:33-34,
  :46-76), which is not this function.
* ``rope_scale``: cos and sin multiplied by the rotary embedding's
  ``attention_scaling`` (models/llama/modeling_llama.py,
  LlamaRotaryEmbedding.forward: ``cos = emb.cos() * self.attention_scaling``).

The reference's fused backward kernel (fused_norm_qkv_rope.py:99-126) is a
plain RMSNorm backward that never applies the transposed rotation, so it is
not the gradient of its forward. ``norm_rope_table_reference_bwd`` restates
that kernel as it is (used only to pin the golden vectors); every parity
check uses the autograd gradient instead.
"""
from __future__ import annotations

import math

import torch

F64 = torch.float64


# ----------------------------------------------------------------- helpers
def inv_freq(head_dim: int, base: float) -> torch.Tensor:
    """inv_freq [head_dim/2] float32 - bloth/bloth/ops/rope.py:71."""
    half = head_dim // 2
    return 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))


def rope_cos_sin(positions: torch.Tensor, inv_f: torch.Tensor, compute=F64):
    """cos/sin [..., D/2] for integer positions - bloth/bloth/ops/rope.py:73-75.

    The angle ``float32(pos) * inv_freq`` is formed in float32 (as
    ``torch.outer(t, inv_freq)`` does with float32 ``t``); cos and sin of that
    float32 angle are then evaluated in ``compute`` precision.
    """
    ang = positions.to(torch.float32).unsqueeze(-1) * inv_f.to(torch.float32)
    ang = ang.to(compute)
    return torch.cos(ang), torch.sin(ang)


def _rms_core(x: torch.Tensor, w: torch.Tensor, eps: float):
    ms = (x * x).mean(-1, keepdim=True)
    rstd = 1.0 / torch.sqrt(ms + eps)
    return x * rstd * w, rstd.squeeze(-1)


def _rotate(n: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, half: int):
    """Rotate-half on the first 2*half columns of n (last dim)."""
    n1 = n[..., :half]
    n2 = n[..., half : 2 * half]
    rest = n[..., 2 * half :]
    y1 = n1 * cos - n2 * sin
    y2 = n1 * sin + n2 * cos
    return torch.cat([y1, y2, rest], dim=-1)


# ------------------------------------------------------------------ RMSNorm
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, compute=F64,
             w_offset: float = 0.0):
    """(y in x.dtype, rstd float32) - bloth/tests/test_kernels.py:124-127."""
    y, rstd = _rms_core(x.to(compute), w.to(compute) + w_offset, eps)
    return y.to(x.dtype), rstd.to(torch.float32)


def rms_norm_fwd_bwd(x, w, dy, eps: float = 1e-6, compute=F64, w_offset: float = 0.0):
    """Forward plus the autograd backward of :func:`rms_norm`.

    Returns y, rstd, dx (x.dtype), dw (w.dtype). The gradient equals the
    reference's manual backward bloth/bloth/kernels/rms_norm.py:101-111.
    """
    xc = x.detach().to(compute).requires_grad_(True)
    wc = w.detach().to(compute).requires_grad_(True)
    y, rstd = _rms_core(xc, wc + w_offset, eps)
    y.backward(dy.to(compute))
    return (y.detach().to(x.dtype), rstd.detach().to(torch.float32),
            xc.grad.to(x.dtype), wc.grad.to(w.dtype))


# --------------------------------------------- residual add + RMSNorm
def add_rms_norm_fwd_bwd(x, r, w, dy, dz_out=None, eps: float = 1e-6, compute=F64,
                         w_offset: float = 0.0):
    """Residual add then RMSNorm, as HF's decoder layer writes them
    (transformers models/llama/modeling_llama.py, LlamaDecoderLayer.forward:
    ``hidden_states = residual + hidden_states`` in the activations' dtype,
    then ``post_attention_layernorm``), with the RMSNorm of :func:`rms_norm`;
    forward and exact backward.

    Returns y, z (x.dtype), rstd, dz (the gradient of both x and r; x.dtype)
    and dw (w.dtype). dz_out is z's gradient from the residual stream (None:
    zero).
    """
    xc = x.detach().to(compute).requires_grad_(True)
    rc = r.detach().to(compute).requires_grad_(True)
    wc = w.detach().to(compute).requires_grad_(True)
    # torch adds 16-bit tensors in fp32 and rounds once to their dtype
    z = (xc.float() + rc.float()).to(x.dtype).to(compute)
    y, rstd = _rms_core(z, wc + w_offset, eps)
    outs, grads = [y], [dy.to(compute)]
    if dz_out is not None:
        outs.append(z)
        grads.append(dz_out.to(compute))
    torch.autograd.backward(outs, grads)
    return (y.detach().to(x.dtype), z.detach().to(x.dtype), rstd.detach().to(torch.float32),
            xc.grad.to(x.dtype), wc.grad.to(w.dtype))


# -------------------------------------------- fused norm + RoPE, row tables
def norm_rope_table(x, w, cos, sin, eps: float = 1e-6, compute=F64):
    """Reference fused_norm_rope forward - fused_norm_qkv_rope.py:59-96.

    x [M, N]; cos, sin [M, h]; returns (y in x.dtype, rstd float32).
    """
    half = cos.shape[-1]
    n, rstd = _rms_core(x.to(compute), w.to(compute), eps)
    y = _rotate(n, cos.to(compute), sin.to(compute), half)
    return y.to(x.dtype), rstd.to(torch.float32)


def norm_rope_table_fwd_bwd(x, w, cos, sin, dy, eps: float = 1e-6, compute=F64):
    """Forward and the exact (autograd) backward of :func:`norm_rope_table`."""
    half = cos.shape[-1]
    xc = x.detach().to(compute).requires_grad_(True)
    wc = w.detach().to(compute).requires_grad_(True)
    n, rstd = _rms_core(xc, wc, eps)
    y = _rotate(n, cos.to(compute), sin.to(compute), half)
    y.backward(dy.to(compute))
    return (y.detach().to(x.dtype), rstd.detach().to(torch.float32),
            xc.grad.to(x.dtype), wc.grad.to(w.dtype))


def norm_rope_table_reference_bwd(x, w, rstd, dy, compute=F64):
    """The reference's fused backward kernel as written -
    bloth/bloth/kernels/fused_norm_qkv_rope.py:115-125: a plain RMSNorm
    backward on dy (no transposed rotation). Not a gradient of the fused
    forward; kept only to pin the reference's golden vectors.
    """
    xc, wc, dyc = x.to(compute), w.to(compute), dy.to(compute)
    r = rstd.to(compute).unsqueeze(-1)
    x_norm = xc * r
    dy_w = dyc * wc
    dot = (dy_w * x_norm).sum(-1, keepdim=True) / x.shape[-1]
    dx = r * (dy_w - x_norm * dot)
    dw = (dyc * x_norm).sum(0)
    return dx.to(x.dtype), dw.to(w.dtype)


# ------------------------------------- per-head q/k norm + RoPE (positions)
def _head_cos_sin(pos, inv_f, cos_tab, sin_tab, compute, D, scale: float = 1.0):
    """cos/sin [B, S, 1, D/2] from positions and inv_freq, or from tables,
    multiplied by ``scale``."""
    if cos_tab is not None:
        c, s = cos_tab[..., : D // 2], sin_tab[..., : D // 2]
        if c.dim() == 2:  # [P, D/2] indexed by position
            c, s = c[pos], s[pos]
        c, s = c.to(compute), s.to(compute)
    else:
        c, s = rope_cos_sin(pos, inv_f, compute)
    return (c * scale).unsqueeze(-2), (s * scale).unsqueeze(-2)


def _positions(B: int, S: int, position_ids, device=None):
    if position_ids is None:
        return torch.arange(S, dtype=torch.int64, device=device).expand(B, S)
    p = position_ids.to(torch.int64)
    if p.dim() == 1:
        p = p.unsqueeze(0)
    return p.expand(B, S)


def qk_norm_rope(q, k, wq, wk, position_ids=None, inv_f=None, eps: float = 1e-6,
                 cos=None, sin=None, compute=F64, w_offset: float = 0.0,
                 rope_scale: float = 1.0):
    """Per-head RMSNorm then rotate-half RoPE for q [B,S,Hq,D] and k [B,S,Hk,D].

    Per (token, head) row this is exactly :func:`norm_rope_table` with
    h = D/2 and that token's cos/sin (fused_norm_qkv_rope.py:59-96); the
    tables follow bloth/bloth/ops/rope.py:71-75. Returns (q_out, k_out, rstd_q,
    rstd_k); rstd are float32 [B, S, H].
    """
    B, S, _, D = q.shape
    pos = _positions(B, S, position_ids, q.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D, rope_scale)
    outs = []
    for x, w in ((q, wq), (k, wk)):
        if x is None:
            outs.append((None, None))
            continue
        n, rstd = _rms_core(x.to(compute), w.to(compute) + w_offset, eps)
        outs.append((_rotate(n, c, s, D // 2).to(x.dtype), rstd.to(torch.float32)))
    return outs[0][0], outs[1][0], outs[0][1], outs[1][1]


def qk_norm_rope_fwd_bwd(q, k, wq, wk, dq_out, dk_out, position_ids=None, inv_f=None,
                         eps: float = 1e-6, cos=None, sin=None, compute=F64,
                         w_offset: float = 0.0, rope_scale: float = 1.0):
    """Forward and exact backward of :func:`qk_norm_rope`.

    Returns dict with q_out, k_out, rstd_q, rstd_k, dq, dk, dwq, dwk.
    """
    B, S, _, D = q.shape
    pos = _positions(B, S, position_ids, q.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D, rope_scale)
    res = {}
    for name, x, w, g in (("q", q, wq, dq_out), ("k", k, wk, dk_out)):
        if x is None:
            continue
        xc = x.detach().to(compute).requires_grad_(True)
        wc = w.detach().to(compute).requires_grad_(True)
        n, rstd = _rms_core(xc, wc + w_offset, eps)
        y = _rotate(n, c, s, D // 2)
        y.backward(g.to(compute))
        res[name + "_out"] = y.detach().to(x.dtype)
        res["rstd_" + name] = rstd.detach().to(torch.float32)
        res["d" + name] = xc.grad.to(x.dtype)
        res["dw" + name] = wc.grad.to(w.dtype)
    return res


# ----------------------------------------------------------------- RoPE only
def rope(x, position_ids=None, inv_f=None, cos=None, sin=None, compute=F64,
         out_dtype=None, rope_scale: float = 1.0):
    """Rotate-half RoPE of x [B, S, H, D] - bloth/bloth/ops/rope.py:21-27."""
    B, S, _, D = x.shape
    pos = _positions(B, S, position_ids, x.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D, rope_scale)
    y = _rotate(x.to(compute), c, s, D // 2)
    return y.to(out_dtype or x.dtype)


def rope_fwd_bwd(x, dy, position_ids=None, inv_f=None, cos=None, sin=None, compute=F64,
                 rope_scale: float = 1.0):
    """RoPE forward and its exact backward (the transposed rotation)."""
    B, S, _, D = x.shape
    pos = _positions(B, S, position_ids, x.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D, rope_scale)
    xc = x.detach().to(compute).requires_grad_(True)
    y = _rotate(xc, c, s, D // 2)
    y.backward(dy.to(compute))
    return y.detach().to(x.dtype), xc.grad.to(x.dtype)


# ------------------------------------------------------------ packed inputs
def packed_position_ids(rows: int, tokens: int, lo: int, hi: int, generator) -> torch.Tensor:
    """Position ids [rows, tokens] of packed documents.

    Each row is filled with documents whose lengths are drawn uniformly from
    [lo, hi] until the remainder is <= hi; the remainder becomes the last
    document if it is >= lo, otherwise the row is redrawn. Positions restart
    at 0 at every document start.
    """
    out = torch.empty(rows, tokens, dtype=torch.int64)
    for r in range(rows):
        while True:
            lens, left = [], tokens
            while left > hi:
                n = int(torch.randint(lo, hi + 1, (1,), generator=generator))
                lens.append(n)
                left -= n
            if left >= lo:
                lens.append(left)
                break
        out[r] = torch.cat([torch.arange(n, dtype=torch.int64) for n in lens])
    return out


def rms_norm_dw_scale(x, dy, eps: float = 1e-6, compute=F64):
    """Per-column root-sum-square of the weight-gradient terms dy * xhat.

    The error of any fp32 evaluation of dweight = sum_rows(dy * xhat) grows
    with this quantity (each term carries a relative rounding error), not
    with |dweight|, which can be far smaller after cancellation.
    """
    xc = x.to(compute)
    rstd = 1.0 / torch.sqrt((xc * xc).mean(-1, keepdim=True) + eps)
    t = dy.to(compute) * xc * rstd
    return torch.sqrt((t * t).reshape(-1, x.shape[-1]).sum(0))


def qk_dw_scale(x, dy, position_ids=None, inv_f=None, eps: float = 1e-6, cos=None, sin=None,
                compute=F64):
    """Per-column root-sum-square of the terms (R^T dy) * xhat of a head
    tensor's weight gradient (see :func:`rms_norm_dw_scale`)."""
    B, S, _, D = x.shape
    pos = _positions(B, S, position_ids, x.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D)
    g = dy.to(compute)
    h = D // 2
    g1, g2 = g[..., :h], g[..., h:]
    dn = torch.cat([g1 * c + g2 * s, g2 * c - g1 * s], -1)
    xc = x.to(compute)
    rstd = 1.0 / torch.sqrt((xc * xc).mean(-1, keepdim=True) + eps)
    t = dn * xc * rstd
    return torch.sqrt((t * t).reshape(-1, D).sum(0))


def norm_rope_table_dw_scale(x, cos, sin, dy, eps: float = 1e-6, compute=F64):
    """Per-column root-sum-square of the weight-gradient terms (R^T dy) * xhat
    of :func:`norm_rope_table` (per-row tables; columns >= 2*half are not
    rotated). See :func:`rms_norm_dw_scale`."""
    h = cos.shape[-1]
    g = dy.to(compute)
    c, s = cos.to(compute), sin.to(compute)
    g1, g2 = g[..., :h], g[..., h:2 * h]
    dn = torch.cat([g1 * c + g2 * s, g2 * c - g1 * s, g[..., 2 * h:]], -1)
    xc = x.to(compute)
    rstd = 1.0 / torch.sqrt((xc * xc).mean(-1, keepdim=True) + eps)
    t = dn * xc * rstd
    return torch.sqrt((t * t).reshape(-1, x.shape[-1]).sum(0))


def rms_norm_dx_scale(x, w, dy, eps: float = 1e-6, compute=F64, dy_mag=None):
    """Elementwise operand magnitude of dx = rstd * (dy*w - xhat*dot):
    rstd * (|dy|*|w| + |xhat*dot|). An fp32 evaluation of the difference
    carries an error proportional to this, which rows of zeros
    (rstd = 1/sqrt(eps)) amplify far beyond |dx|. ``dy_mag`` replaces |dy|
    when dy is itself a sum (the rotated gradient of the fused op)."""
    xc, wc = x.to(compute), w.to(compute)
    g = dy.to(compute) * wc
    rstd = 1.0 / torch.sqrt((xc * xc).mean(-1, keepdim=True) + eps)
    xh = xc * rstd
    dot = (g * xh).mean(-1, keepdim=True)
    mag = dy.to(compute).abs() if dy_mag is None else dy_mag
    return rstd * (mag * wc.abs() + (xh * dot).abs())


def qk_dx_scale(x, w, dy, position_ids=None, inv_f=None, eps: float = 1e-6, cos=None,
                sin=None, compute=F64):
    """:func:`rms_norm_dx_scale` for a head tensor: dy is rotated back
    (dn = R^T dy), and |dn| is replaced by the magnitude of its two terms."""
    B, S, _, D = x.shape
    pos = _positions(B, S, position_ids, x.device)
    c, s = _head_cos_sin(pos, inv_f, cos, sin, compute, D)
    g = dy.to(compute)
    h = D // 2
    g1, g2 = g[..., :h], g[..., h:]
    dn = torch.cat([g1 * c + g2 * s, g2 * c - g1 * s], -1)
    mag = torch.cat([(g1 * c).abs() + (g2 * s).abs(), (g2 * c).abs() + (g1 * s).abs()], -1)
    return rms_norm_dx_scale(x, w, dn, eps, compute, dy_mag=mag)


def tolerance_ok(got: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype,
                 scale_with_magnitude: bool = False, scale: torch.Tensor | None = None
                 ) -> tuple[bool, float]:
    """Elementwise tolerance of the path: fp32 max abs <= 1e-5; bf16/fp16 abs
    <= 2e-2 or rel <= 1.6e-2. With ``scale_with_magnitude`` the fp32 bound
    becomes 1e-5 * max(1, |ref|) (values whose magnitude puts 1e-5 below
    fp32 resolution, e.g. weight gradients summed over millions of rows, or
    rows of zeros where rstd = 1/sqrt(eps)); ``scale`` (a per-element
    magnitude, e.g. :func:`rms_norm_dw_scale` for a weight gradient) raises
    the fp32 bound to at least 1e-5 * scale. Returns (ok, worst excess).
    """
    g = got.to(F64)
    r = ref.to(F64)
    err = (g - r).abs()
    if dtype == torch.float32:
        bound = 1e-5 * (torch.clamp(r.abs(), min=1.0) if scale_with_magnitude else 1.0)
        if scale is not None:
            bound = torch.maximum(torch.as_tensor(bound, dtype=F64, device=r.device),
                                  1e-5 * scale.to(F64).to(r.device))
        excess = (err - bound)
    else:
        rel = err / r.abs().clamp(min=1e-30)
        ok_el = (err <= 2e-2) | (rel <= 1.6e-2)
        excess = torch.where(ok_el, torch.zeros_like(err), err)
    worst = float(excess.max()) if excess.numel() else 0.0
    finite = bool(torch.isfinite(g).all())
    return (worst <= 0.0 and finite), worst


def seeded_normal(shape, dtype, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float32).to(dtype)


def seeded_weight(n: int, dtype, seed: int) -> torch.Tensor:
    """weight = 1 + 0.1 * N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(n, generator=g, dtype=torch.float32)).to(dtype)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "torch")]
