"""The bandwidth/precision sweep config at its larger points: hidden rows of
8192 and q/k 32 + 8 heads of 128, bf16 and fp32, inputs ~N(0,1) with 1% of
elements x100 and ~0.1% of rows all zeros, fwd + bwd.

2^16 and 2^18 tokens are checked in full against the oracle, evaluated in
float64 on the GPU over row chunks (rows are independent; weight gradients
sum over the chunks). 2^22 tokens (bf16) run as the sweep runs them, four
chunks of 2^20 tokens through the same device buffers: each chunk's sampled
tokens are checked against the CPU oracle, and the weight gradients summed
over the chunks against the float64 oracle of all 2^22 tokens.

Tolerances are the path's (oracle.tolerance_ok): fp32 max abs 1e-5, raised
to 1e-5 x the operand magnitude where the exact value is a long sum or a
difference (oracle.*_dw_scale, oracle.*_dx_scale); bf16 abs <= 2e-2 or rel
<= 1.6e-2.
"""
import pytest
import torch

import bloth_b200
import oracle
from oracle.reference_path import tolerance_ok

pytestmark = pytest.mark.gpu
F64 = torch.float64
HD, HQ, HK, D, EPS = 8192, 32, 8, 128, 1e-5


def _stress(shape, dtype, gen, dev):
    """N(0,1), 1% of elements x100, ~0.1% of rows (>= 1) all zeros; made on
    the device."""
    t = torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32)
    t[torch.rand(*shape, generator=gen, device=dev) < 0.01] *= 100
    rows = t.view(-1, shape[-1])
    nz = max(1, rows.shape[0] // 1000)
    rows[torch.randperm(rows.shape[0], generator=gen, device=dev)[:nz]] = 0
    return t.to(dtype)


def _weight(n, dtype, gen, dev):
    return (1 + 0.1 * torch.randn(n, generator=gen, device=dev)).to(dtype)


def _assert(got, ref, dtype, what, scale=None):
    ok, worst = tolerance_ok(got, ref, dtype, scale_with_magnitude=True, scale=scale)
    assert ok, f"{what}: worst excess over tolerance {worst:.3e}"


def _hidden(x, w, g):
    """Forward and backward through the public op; fresh leaves every call,
    so reused buffers never accumulate gradients."""
    x = x.detach().requires_grad_(True)
    w = w.detach().clone().requires_grad_(True)
    y = bloth_b200.rms_norm(x, w, EPS)
    dx, dw = torch.autograd.grad(y, (x, w), g)
    return y.detach(), dx, dw


def _qk(q, k, wq, wk, gq, gk, inv):
    q, k = q.detach().requires_grad_(True), k.detach().requires_grad_(True)
    wq = wq.detach().clone().requires_grad_(True)
    wk = wk.detach().clone().requires_grad_(True)
    qo, ko = bloth_b200.fused_qk_norm_rope(q, k, wq, wk, None, inv, EPS)
    dq, dk, dwq, dwk = torch.autograd.grad([qo, ko], [q, k, wq, wk], [gq, gk])
    return {"q_out": qo.detach(), "k_out": ko.detach(), "dq": dq, "dk": dk, "dwq": dwq,
            "dwk": dwk}


def _fill_stress(buf, gen):
    """_stress into an existing buffer, a slab of rows at a time (bounded
    temporaries for the largest chunks)."""
    rows = buf.view(-1, buf.shape[-1])
    slab = 1 << 16
    for s in range(0, rows.shape[0], slab):
        part = rows[s:s + slab]
        part.copy_(_stress(tuple(part.shape), torch.float32, gen, part.device))


def _fill_normal(buf, gen):
    rows = buf.view(-1, buf.shape[-1])
    slab = 1 << 16
    for s in range(0, rows.shape[0], slab):
        part = rows[s:s + slab]
        part.copy_(torch.randn(*part.shape, generator=gen, device=part.device))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("lg", [16, 18])
def test_c5_full_check(cuda, dtype, lg):
    T = 1 << lg
    gen = torch.Generator(device=cuda).manual_seed(lg)
    chunk = 1 << 14
    # hidden rows of 8192
    x = _stress((T, HD), dtype, gen, cuda)
    w = _weight(HD, dtype, gen, cuda)
    g = torch.randn(T, HD, generator=gen, device=cuda).to(dtype)
    y, dx, dw = _hidden(x, w, g)
    dw_ref = torch.zeros(HD, dtype=F64, device=cuda)
    dw_sq = torch.zeros(HD, dtype=F64, device=cuda)
    for s in range(0, T, chunk):
        sl = slice(s, s + chunk)
        ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x[sl], w.to(F64), g[sl], EPS)
        _assert(y[sl], ry, dtype, f"2^{lg} {dtype} hidden y")
        _assert(dx[sl], rdx, dtype, f"2^{lg} {dtype} hidden dx",
                oracle.rms_norm_dx_scale(x[sl], w, g[sl], EPS))
        dw_ref += rdw
        dw_sq += oracle.rms_norm_dw_scale(x[sl], g[sl], EPS) ** 2
    _assert(dw, dw_ref, dtype, f"2^{lg} {dtype} hidden dw", dw_sq.sqrt())
    del x, g, y, dx
    # q/k 32 + 8 heads of 128, positions 0..T-1
    q = _stress((1, T, HQ, D), dtype, gen, cuda)
    k = _stress((1, T, HK, D), dtype, gen, cuda)
    wq, wk = _weight(D, dtype, gen, cuda), _weight(D, dtype, gen, cuda)
    gq = torch.randn(1, T, HQ, D, generator=gen, device=cuda).to(dtype)
    gk = torch.randn(1, T, HK, D, generator=gen, device=cuda).to(dtype)
    inv = oracle.inv_freq(D, 5e5).to(cuda)
    res = _qk(q, k, wq, wk, gq, gk, inv)
    acc = {key: torch.zeros(D, dtype=F64, device=cuda) for key in ("dwq", "dwk")}
    sq = {key: torch.zeros(D, dtype=F64, device=cuda) for key in ("dwq", "dwk")}
    for s in range(0, T, chunk):
        sl = slice(s, s + chunk)
        pos = torch.arange(s, s + chunk, device=cuda).view(1, -1)
        ref = oracle.qk_norm_rope_fwd_bwd(q[:, sl], k[:, sl], wq.to(F64), wk.to(F64), gq[:, sl],
                                          gk[:, sl], pos, inv, EPS)
        for key in ("q_out", "k_out"):
            _assert(res[key][:, sl], ref[key], dtype, f"2^{lg} {dtype} {key}")
        for key, xx, ww, gg in (("dq", q, wq, gq), ("dk", k, wk, gk)):
            _assert(res[key][:, sl], ref[key], dtype, f"2^{lg} {dtype} {key}",
                    oracle.qk_dx_scale(xx[:, sl], ww, gg[:, sl], pos, inv, EPS))
        for key, xx, gg in (("dwq", q, gq), ("dwk", k, gk)):
            acc[key] += ref[key]
            sq[key] += oracle.qk_dw_scale(xx[:, sl], gg[:, sl], pos, inv, EPS) ** 2
    for key in ("dwq", "dwk"):
        _assert(res[key], acc[key], dtype, f"2^{lg} {dtype} {key}", sq[key].sqrt())
    assert bloth_b200.device_fault() == 0


def test_c5_chunked_2e22_bf16_sampled(cuda):
    dtype, T, CH = torch.bfloat16, 1 << 22, 1 << 20
    gen = torch.Generator(device=cuda).manual_seed(22)
    cpu_gen = torch.Generator().manual_seed(22)
    inv = oracle.inv_freq(D, 5e5).to(cuda)
    w = _weight(HD, dtype, gen, cuda)
    wq, wk = _weight(D, dtype, gen, cuda), _weight(D, dtype, gen, cuda)
    dw_sum = {key: torch.zeros(n, dtype=F64, device=cuda)
              for key, n in (("dw", HD), ("dwq", D), ("dwk", D))}
    dw_mag = {key: torch.zeros_like(v) for key, v in dw_sum.items()}
    dw_ref = {key: torch.zeros_like(v) for key, v in dw_sum.items()}
    # one set of device buffers, refilled for every chunk (as the sweep runs)
    x = torch.empty(CH, HD, dtype=dtype, device=cuda)
    g = torch.empty_like(x)
    q = torch.empty(1, CH, HQ, D, dtype=dtype, device=cuda)
    k = torch.empty(1, CH, HK, D, dtype=dtype, device=cuda)
    gq, gk = torch.empty_like(q), torch.empty_like(k)
    for c in range(T // CH):
        _fill_stress(x, gen)
        _fill_normal(g, gen)
        _fill_stress(q, gen)
        _fill_stress(k, gen)
        _fill_normal(gq, gen)
        _fill_normal(gk, gen)
        y, dx, dw = _hidden(x, w, g)
        # positions 0..CH-1 in every chunk (position_ids None)
        res = _qk(q, k, wq, wk, gq, gk, inv)
        pos = torch.arange(CH, device=cuda).view(1, -1)
        # sampled tokens against the CPU oracle
        idx = torch.randperm(CH, generator=cpu_gen)[:48]
        s = lambda t: t[idx.to(t.device)].cpu()  # noqa: E731
        ry, _, rdx, _ = oracle.rms_norm_fwd_bwd(s(x), w.cpu(), s(g), EPS)
        _assert(s(y), ry, dtype, f"chunk {c} hidden y")
        _assert(s(dx), rdx, dtype, f"chunk {c} hidden dx")
        sq = lambda t: t[0, idx.to(t.device)].unsqueeze(0).cpu()  # noqa: E731
        ref = oracle.qk_norm_rope_fwd_bwd(sq(q), sq(k), wq.cpu(), wk.cpu(), sq(gq), sq(gk),
                                          idx.view(1, -1), inv.cpu(), EPS)
        for key in ("q_out", "k_out", "dq", "dk"):
            _assert(sq(res[key]), ref[key], dtype, f"chunk {c} {key}")
        # weight gradients: this chunk's kernel result and its float64 oracle
        for key, got in (("dw", dw), ("dwq", res["dwq"]), ("dwk", res["dwk"])):
            dw_sum[key] += got.double()
            dw_mag[key] += got.double().abs()
        for s0 in range(0, CH, 1 << 16):
            sl = slice(s0, s0 + (1 << 16))
            dw_ref["dw"] += oracle.rms_norm_fwd_bwd(x[sl], w.to(F64), g[sl], EPS)[3]
            r = oracle.qk_norm_rope_fwd_bwd(q[:, sl], k[:, sl], wq.to(F64), wk.to(F64),
                                            gq[:, sl], gk[:, sl], pos[:, sl], inv, EPS)
            dw_ref["dwq"] += r["dwq"]
            dw_ref["dwk"] += r["dwk"]
        del y, dx, dw, res
    # each chunk's dweight is rounded to bf16 before the sum over chunks, so
    # the bf16 rule applies to the sum of the chunks' magnitudes
    for key in dw_sum:
        err = (dw_sum[key] - dw_ref[key]).abs()
        bound = torch.clamp(1.6e-2 * dw_mag[key], min=2e-2)
        assert bool((err <= bound).all()), f"2^22 {key}: worst {float((err - bound).max()):.3e}"
    assert bloth_b200.device_fault() == 0
