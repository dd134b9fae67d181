"""The contiguous q/k path of fused_qk_norm_rope: q [B, S, Hq, D] and k
[B, S, Hk, D] computed in token blocks (a block holds the q and the k rows of
1-8 consecutive tokens, moved by one bulk copy per tensor; a thread holds a
column and its rotation partner; the block's cos/sin are evaluated once in
shared memory and shared by q and k).

The token-block kernels take a call when every head tensor is contiguous and
cos/sin come from inv_freq; the backward also needs head counts that are
multiples of 4 (each block's rstd run is then a 16-byte unit). Cases here
cover every head dim and element type, blocks of one to several tokens,
partial last blocks, head counts that are not multiples of 4 (token-block
forward, per-head backward), q without k, weight offset, rope scale, int32
and broadcast positions, positions that restart per document, a whole wave of
CTAs with the workspace the library reports, bit-identical reruns, and
agreement with the per-head kernel (which takes the same tensors when they
are strided views). Tolerances are the path's (oracle.tolerance_ok): fp32 max
abs 1e-5 (1e-5 x magnitude for weight gradients summed over many rows),
bf16/fp16 abs <= 2e-2 or rel <= 1.6e-2.
"""
import pytest
import torch

import bloth_b200
import oracle
from oracle.reference_path import seeded_normal, seeded_weight, tolerance_ok

pytestmark = pytest.mark.gpu


def _inputs(B, S, Hq, Hk, D, dtype, dev, seed, wdtype=None):
    wdtype = wdtype or dtype
    q = seeded_normal((B, S, Hq, D), dtype, seed).to(dev)
    k = seeded_normal((B, S, Hk, D), dtype, seed + 1).to(dev) if Hk else None
    wq = seeded_weight(D, wdtype, seed + 2).to(dev)
    wk = seeded_weight(D, wdtype, seed + 3).to(dev) if Hk else None
    gq = seeded_normal((B, S, Hq, D), dtype, seed + 4).to(dev)
    gk = seeded_normal((B, S, Hk, D), dtype, seed + 5).to(dev) if Hk else None
    return q, k, wq, wk, gq, gk


def _run(q, k, wq, wk, gq, gk, pos, inv, eps, w_off=0.0, scale=1.0):
    q = q.detach().clone().requires_grad_(True)
    wq = wq.detach().clone().requires_grad_(True)
    k = None if k is None else k.detach().clone().requires_grad_(True)
    wk = None if wk is None else wk.detach().clone().requires_grad_(True)
    out = bloth_b200.fused_qk_norm_rope(q, k, wq, wk, pos, inv, eps, weight_offset=w_off,
                                        rope_scale=scale)
    out = (out,) if k is None else out
    torch.autograd.backward(out, (gq,) if k is None else (gq, gk))
    torch.cuda.synchronize()
    res = {"q_out": out[0], "dq": q.grad, "dwq": wq.grad}
    if k is not None:
        res.update(k_out=out[1], dk=k.grad, dwk=wk.grad)
    return res


def _check(res, q, k, wq, wk, gq, gk, pos, inv, eps, dtype, w_off=0.0, scale=1.0, what=""):
    B, S = q.shape[:2]
    p = None if pos is None else pos.long().expand(B, S).cpu()
    t = lambda x: None if x is None else x.cpu()  # noqa: E731
    ref = oracle.qk_norm_rope_fwd_bwd(t(q), t(k), t(wq), t(wk), t(gq), t(gk), p, inv.cpu(), eps,
                                      w_offset=w_off, rope_scale=scale)
    for key in ("q_out", "k_out", "dq", "dk"):
        if key in res:
            ok, worst = tolerance_ok(res[key].detach().cpu(), ref[key], dtype)
            assert ok, f"{what}{key}: worst excess {worst:.3e}"
    for key, x, g in (("dwq", q, gq), ("dwk", k, gk)):
        if key in res:
            ok, worst = tolerance_ok(res[key].detach().cpu(), ref[key], dtype,
                                     scale_with_magnitude=True,
                                     scale=oracle.qk_dw_scale(x.cpu(), g.cpu(), p, inv.cpu(), eps))
            assert ok, f"{what}{key}: worst excess {worst:.3e}"


# (B, S, Hq, Hk, D, dtype): tokens per block follow from ~20 KB of rows per
# block (1 to 8 here); odd token counts leave a partial last block; 5/3 and
# 6/2 heads take the token-block forward and the per-head backward.
CASES = [
    (1, 37, 32, 8, 128, torch.bfloat16),
    (2, 19, 16, 8, 256, torch.bfloat16),
    (1, 37, 12, 12, 64, torch.bfloat16),
    (2, 23, 32, 16, 64, torch.float16),
    (1, 45, 8, 4, 128, torch.float32),
    (1, 33, 4, 4, 64, torch.float32),
    (1, 21, 8, 4, 256, torch.float32),
    (1, 29, 64, 8, 128, torch.bfloat16),
    (3, 7, 5, 3, 128, torch.bfloat16),
    (1, 13, 6, 2, 64, torch.float32),
]


@pytest.mark.parametrize("B,S,Hq,Hk,D,dtype", CASES)
def test_token_blocks_layouts(cuda, B, S, Hq, Hk, D, dtype):
    q, k, wq, wk, gq, gk = _inputs(B, S, Hq, Hk, D, dtype, cuda, seed=D + Hq)
    inv = oracle.inv_freq(D, 5e5).to(cuda)
    pos = torch.randint(0, 9000, (B, S), generator=torch.Generator().manual_seed(2)).to(cuda)
    res = _run(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    _check(res, q, k, wq, wk, gq, gk, pos, inv, 1e-6, dtype, what=f"{D} {dtype} ")
    assert bloth_b200.device_fault() == 0


def test_token_blocks_options(cuda):
    # fp32 weights with fp16 tensors, weight offset, rope scale, int32
    # positions broadcast over the batch, and q without k
    dt = torch.float16
    q, k, wq, wk, gq, gk = _inputs(3, 29, 16, 8, 128, dt, cuda, seed=70, wdtype=torch.float32)
    inv = oracle.inv_freq(128, 1e6).to(cuda)
    pos = torch.arange(5, 34, dtype=torch.int32, device=cuda).view(1, 29)
    res = _run(q, k, wq, wk, gq, gk, pos, inv, 1e-5, w_off=1.0, scale=0.7)
    _check(res, q, k, wq, wk, gq, gk, pos, inv, 1e-5, dt, w_off=1.0, scale=0.7, what="opts ")
    assert res["dwq"].dtype == torch.float32
    res = _run(q, None, wq, None, gq, None, pos, inv, 1e-5)
    _check(res, q, None, wq, None, gq, None, pos, inv, 1e-5, dt, what="q only ")
    # positions default to 0..S-1
    res = _run(q, k, wq, wk, gq, gk, None, inv, 1e-5)
    _check(res, q, k, wq, wk, gq, gk, torch.arange(29, device=cuda).view(1, 29), inv, 1e-5, dt,
           what="no pos ")


def test_token_blocks_packed_documents(cuda):
    dt = torch.bfloat16
    B, S = 2, 3000
    pos = oracle.packed_position_ids(B, S, 64, 2048, torch.Generator().manual_seed(5)).to(cuda)
    q, k, wq, wk, gq, gk = _inputs(B, S, 32, 8, 128, dt, cuda, seed=80)
    inv = oracle.inv_freq(128, 1e6).to(cuda)
    res = _run(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    _check(res, q, k, wq, wk, gq, gk, pos, inv, 1e-6, dt, what="packed ")


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.bfloat16),
                                     (128, torch.float32)])
def test_token_blocks_full_wave_and_reruns(cuda, D, dtype):
    # more blocks than one wave of the backward holds (148 SMs x resident
    # CTAs), through the workspace size the library reports; then the same
    # call again, bit for bit
    B, S, Hq, Hk = 1, 1027, 32, 8
    q, k, wq, wk, gq, gk = _inputs(B, S, Hq, Hk, D, dtype, cuda, seed=90)
    inv = oracle.inv_freq(D, 5e5).to(cuda)
    pos = torch.arange(S, device=cuda).view(1, S)
    res = _run(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    eps = 1e-6
    ref = oracle.qk_norm_rope_fwd_bwd(q, k, wq, wk, gq, gk, pos.expand(B, S), inv, eps)  # GPU f64
    for key in ("q_out", "k_out", "dq", "dk"):
        ok, worst = tolerance_ok(res[key].detach(), ref[key], dtype)
        assert ok, f"{key}: {worst:.3e}"
    for key, x, g in (("dwq", q, gq), ("dwk", k, gk)):
        ok, worst = tolerance_ok(res[key], ref[key], dtype, scale_with_magnitude=True,
                                 scale=oracle.qk_dw_scale(x, g, pos.expand(B, S), inv, eps))
        assert ok, f"{key}: {worst:.3e}"
    again = _run(q, k, wq, wk, gq, gk, pos, inv, eps)
    for key in res:
        assert torch.equal(res[key], again[key]), key


def test_token_blocks_kernel_agrees_with_the_head_kernel(cuda):
    # the same values as strided views (slices of a packed projection) take
    # the per-head kernel; both must meet the tolerance against the oracle
    dt = torch.bfloat16
    B, S, Hq, Hk, D = 2, 41, 32, 8, 128
    qkv = seeded_normal((B, S, Hq + 2 * Hk, D), dt, 100).to(cuda)
    qs, ks = qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hk]
    qc, kc = qs.contiguous(), ks.contiguous()
    wq, wk = seeded_weight(D, dt, 101).to(cuda), seeded_weight(D, dt, 102).to(cuda)
    gq = seeded_normal((B, S, Hq, D), dt, 103).to(cuda)
    gk = seeded_normal((B, S, Hk, D), dt, 104).to(cuda)
    inv = oracle.inv_freq(D, 5e5).to(cuda)
    pos = torch.arange(S, device=cuda).expand(B, S)
    rows = _run(qc, kc, wq, wk, gq, gk, pos, inv, 1e-6)
    heads = _run(qs, ks, wq, wk, gq, gk, pos, inv, 1e-6)
    _check(rows, qc, kc, wq, wk, gq, gk, pos, inv, 1e-6, dt, what="rows ")
    _check(heads, qc, kc, wq, wk, gq, gk, pos, inv, 1e-6, dt, what="heads ")
    for key in ("q_out", "k_out", "dq", "dk"):
        ok, worst = tolerance_ok(rows[key].cpu(), heads[key].cpu().double(), dt)
        assert ok, f"{key}: rows vs heads {worst:.3e}"
