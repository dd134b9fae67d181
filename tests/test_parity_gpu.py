"""GPU parity: the sm_100a kernels (through the public ops, i.e. the C ABI)
against the oracle on seeded inputs, per workload, plus edge cases.

Tolerance (stated per the path's contract): fp32 max abs error <= 1e-5; bf16
and fp16 elementwise abs <= 2e-2 or rel <= 1.6e-2; on outputs, dx/dq/dk and
dweight. Where the exact value's magnitude puts 1e-5 below fp32 resolution
(weight gradients summed over >=2^14 rows, rows of zeros whose rstd is
1/sqrt(eps)), the fp32 bound is 1e-5 * max(1, |exact|), and for quantities
formed as a difference or a long sum it is 1e-5 * the magnitude of the
operands (oracle.*_dx_scale, oracle.*_dw_scale): any fp32 evaluation carries
rounding error proportional to that, not to the possibly much smaller result.

Small workloads run the oracle on the CPU in float64. The full-size
workloads evaluate the same oracle expressions in float64 on the GPU (plain
torch ops, independent of the kernels) and additionally check sampled tokens
against the CPU oracle.
"""
import pytest
import torch

import bloth_b200
import oracle
from oracle.reference_path import tolerance_ok, seeded_normal, seeded_weight
from tests.golden import load

pytestmark = pytest.mark.gpu
F64 = torch.float64


def assert_tol(got, ref, dtype, what, scale=False, dw_scale=None):
    ok, worst = tolerance_ok(got.detach().to(ref.device), ref, dtype, scale_with_magnitude=scale,
                             scale=dw_scale)
    assert ok, f"{what}: worst excess over tolerance {worst:.3e}"


def run_qk(q, k, wq, wk, gq, gk, pos=None, inv=None, eps=1e-6, cos=None, sin=None):
    q = q.detach().clone().requires_grad_(True)
    wq = wq.detach().clone().requires_grad_(True)
    k = None if k is None else k.detach().clone().requires_grad_(True)
    wk = None if wk is None else wk.detach().clone().requires_grad_(True)
    out = bloth_b200.fused_qk_norm_rope(q, k, wq, wk, pos, inv, eps, cos=cos, sin=sin)
    if k is None:
        out = (out,)
        torch.autograd.backward(out, (gq,))
    else:
        torch.autograd.backward(out, (gq, gk))
    torch.cuda.synchronize()
    res = {"q_out": out[0], "dq": q.grad, "dwq": wq.grad}
    if k is not None:
        res.update(k_out=out[1], dk=k.grad, dwk=wk.grad)
    return res


def compare_qk(res, ref, dtype, scale=False, what=""):
    for key in ("q_out", "k_out", "dq", "dk"):
        if key in res:
            assert_tol(res[key], ref[key], dtype, what + key, scale)
    for key in ("dwq", "dwk"):
        if key in res:
            assert_tol(res[key], ref[key], dtype, what + key, True)


def qk_inputs(B, S, Hq, Hk, D, dtype, dev, seed=0, wdtype=None):
    wdtype = wdtype or dtype
    q = seeded_normal((B, S, Hq, D), dtype, seed).to(dev)
    k = seeded_normal((B, S, Hk, D), dtype, seed + 1).to(dev)
    wq = seeded_weight(D, wdtype, seed + 2).to(dev)
    wk = seeded_weight(D, wdtype, seed + 3).to(dev)
    gq = seeded_normal((B, S, Hq, D), dtype, seed + 4).to(dev)
    gk = seeded_normal((B, S, Hk, D), dtype, seed + 5).to(dev)
    return q, k, wq, wk, gq, gk


def oracle_qk(q, k, wq, wk, gq, gk, pos=None, inv=None, eps=1e-6, cos=None, sin=None,
              device="cpu"):
    t = lambda x: None if x is None else x.to(device)  # noqa: E731
    return oracle.qk_norm_rope_fwd_bwd(t(q), t(k), t(wq), t(wk), t(gq), t(gk), t(pos), t(inv),
                                       eps, t(cos), t(sin))


def run_rms(x, w, g, eps):
    x = x.detach().clone().requires_grad_(True)
    w = w.detach().clone().requires_grad_(True)
    y = bloth_b200.rms_norm(x, w, eps)
    y.backward(g)
    torch.cuda.synchronize()
    return y, x.grad, w.grad


# ------------------------------------------------------------------ CPU config
def test_c1_qk_positions_fp32(cuda):
    # q [2,128,8,64], k [2,128,2,64] fp32, eps 1e-6, theta 1e4, positions 0..127
    q, k, wq, wk, gq, gk = qk_inputs(2, 128, 8, 2, 64, torch.float32, cuda)
    inv = oracle.inv_freq(64, 1e4).to(cuda)
    pos = torch.arange(128, device=cuda).expand(2, 128)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    compare_qk(res, ref, torch.float32, what="C1 ")
    # strict 1e-5 on dweight too at this size
    for key in ("dwq", "dwk"):
        assert float((res[key].cpu().double() - ref[key].double()).abs().max()) <= 1e-5, key


def test_c1_reference_signature_fp32(cuda):
    q, k, wq, wk, gq, gk = qk_inputs(2, 128, 8, 2, 64, torch.float32, cuda)
    inv = oracle.inv_freq(64, 1e4)
    cos_t, sin_t = oracle.rope_cos_sin(torch.arange(128), inv, torch.float32)
    for x, w, g, H in ((q, wq, gq, 8), (k, wk, gk, 2)):
        rows = torch.arange(128).view(1, 128, 1).expand(2, 128, H).reshape(-1)
        cos, sin = cos_t[rows], sin_t[rows]
        xr = x.detach().clone().requires_grad_(True)
        wr = w.detach().clone().requires_grad_(True)
        y = bloth_b200.kernels.fused_norm_rope(xr.view(-1, 64), wr, cos.to(cuda), sin.to(cuda), 1e-6)
        y.backward(g.view(-1, 64))
        ry, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(x.cpu().view(-1, 64), w.cpu(), cos, sin,
                                                         g.cpu().view(-1, 64), 1e-6)
        assert_tol(y, ry, torch.float32, "y")
        assert_tol(xr.grad.view(-1, 64), rdx, torch.float32, "dx")
        assert float((wr.grad.cpu().double() - rdw.double()).abs().max()) <= 1e-5


def test_golden_fused_vectors_through_kernel(cuda):
    # the reference's own Triton outputs (interpreter run) for the C1 q and k
    for name, H in (("q", 8), ("k", 2)):
        g = load(f"fused_{name}_f32")
        D = g["x"].shape[-1]
        rows = torch.arange(128).view(1, 128, 1).expand(2, 128, H).reshape(-1)
        y = bloth_b200.kernels.fused_norm_rope(g["x"].to(cuda).view(-1, D), g["w"].to(cuda),
                                               g["cos"][rows].to(cuda), g["sin"][rows].to(cuda),
                                               g["eps"])
        assert float((y.cpu().view_as(g["y"]) - g["y"]).abs().max()) <= 1e-5, name
        # the position form reproduces the same reference vectors
        inv = oracle.inv_freq(D, g["theta"]).to(cuda)
        qo = bloth_b200.fused_qk_norm_rope(g["x"].to(cuda), None, g["w"].to(cuda), None, None,
                                           inv, g["eps"])
        assert float((qo.cpu() - g["y"]).abs().max()) <= 1e-5, name


def test_golden_rmsnorm_vectors_through_kernel(cuda):
    g = load("rmsnorm_f32")
    y, dx, dw = run_rms(g["x"].to(cuda), g["w"].to(cuda), g["dy"].to(cuda), g["eps"])
    assert float((y.cpu() - g["y"]).abs().max()) <= 1e-5
    assert float((dx.cpu() - g["dx"]).abs().max()) <= 1e-5
    assert float((dw.cpu() - g["dw"]).abs().max()) <= 1e-4  # reference: fp32 atomics
    gb = load("rmsnorm_bf16")
    yb = bloth_b200.rms_norm(gb["x"].to(cuda), gb["w"].to(cuda))
    assert_tol(yb.cpu(), gb["y"], torch.bfloat16, "bf16 golden")
    # the reference test's own golden (bloth/tests/test_kernels.py:124-127):
    # the same bf16 value except where the fp32 results straddle a bf16
    # rounding boundary, and never more than one bf16 ulp apart
    x32 = gb["x"].float()
    gold = (x32 / x32.pow(2).mean(-1, keepdim=True).add(1e-6).sqrt() * gb["w"].float()).bfloat16()
    same = (yb.cpu().view(torch.int16) == gold.view(torch.int16)).float().mean()
    assert same > 0.999
    ulp = torch.finfo(torch.bfloat16).eps * gold.float().abs()
    assert bool(((yb.cpu().float() - gold.float()).abs() <= ulp + 1e-30).all())


def test_golden_rope_embedding(cuda):
    g = load("rope_bf16")
    y = bloth_b200.rope_embedding(g["x"].to(cuda), g["cos"].to(cuda), g["sin"].to(cuda))
    assert y.shape == g["x"].shape and y.dtype == torch.bfloat16
    assert_tol(y.cpu(), g["y"], torch.bfloat16, "rope_embedding")
    mod = bloth_b200.BlothRoPE(64, max_seq_len=16, base=1e4).to(cuda)
    assert_tol(mod(g["x"].to(cuda)).cpu(), g["y"], torch.bfloat16, "BlothRoPE")


# --------------------------------------------------------- Llama-3.2-1B shape
def test_c2_llama32_1b_bf16(cuda):
    eps = 1e-5
    x = seeded_normal((4, 2048, 2048), torch.bfloat16, 100).to(cuda)
    w = seeded_weight(2048, torch.bfloat16, 101).to(cuda)
    g = seeded_normal((4, 2048, 2048), torch.bfloat16, 102).to(cuda)
    y, dx, dw = run_rms(x, w, g, eps)
    ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x.cpu(), w.cpu(), g.cpu(), eps)
    assert_tol(y.cpu(), ry, torch.bfloat16, "hidden y")
    assert_tol(dx.cpu(), rdx, torch.bfloat16, "hidden dx")
    assert_tol(dw.cpu(), rdw, torch.bfloat16, "hidden dw")

    q, k, wq, wk, gq, gk = qk_inputs(4, 2048, 32, 8, 64, torch.bfloat16, cuda, seed=110)
    inv = oracle.inv_freq(64, 5e5).to(cuda)
    pos = torch.arange(2048, device=cuda).expand(4, 2048)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv, eps)
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos, inv, eps)
    compare_qk(res, ref, torch.bfloat16, what="C2 ")


# ----------------------------------------------------------- Llama-3-8B shape
def _sample_tokens_cpu_check(res, q, k, wq, wk, gq, gk, pos, inv, eps, dtype, n=64):
    """Rows (tokens) are independent: check a sample of tokens against the CPU
    oracle (dweight excluded, it sums over all tokens)."""
    B, S = q.shape[:2]
    gen = torch.Generator().manual_seed(7)
    flat = torch.randperm(B * S, generator=gen)[:n]
    b, s = flat // S, flat % S
    sel = lambda t: t[b.to(t.device), s.to(t.device)].unsqueeze(0).cpu()  # noqa: E731
    p = None if pos is None else sel(pos)
    ref = oracle.qk_norm_rope_fwd_bwd(sel(q), sel(k), wq.cpu(), wk.cpu(), sel(gq), sel(gk), p,
                                      inv.cpu(), eps)
    for key, full in (("q_out", res["q_out"]), ("k_out", res["k_out"]), ("dq", res["dq"]),
                      ("dk", res["dk"])):
        assert_tol(sel(full.detach()), ref[key], dtype, "sampled " + key)


def test_c3_llama3_8b_bf16_full(cuda):
    eps = 1e-5
    x = seeded_normal((8, 4096, 4096), torch.bfloat16, 200).to(cuda)
    w = seeded_weight(4096, torch.bfloat16, 201).to(cuda)
    g = seeded_normal((8, 4096, 4096), torch.bfloat16, 202).to(cuda)
    y, dx, dw = run_rms(x, w, g, eps)
    ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x, w, g, eps)  # float64 on the GPU
    assert_tol(y, ry, torch.bfloat16, "hidden y")
    assert_tol(dx, rdx, torch.bfloat16, "hidden dx")
    assert_tol(dw, rdw, torch.bfloat16, "hidden dw")
    del x, g, y, dx, ry, rdx

    q, k, wq, wk, gq, gk = qk_inputs(8, 4096, 32, 8, 128, torch.bfloat16, cuda, seed=210)
    inv = oracle.inv_freq(128, 5e5).to(cuda)
    pos = torch.arange(4096, device=cuda).expand(8, 4096)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv, eps)
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos, inv, eps, device=cuda)
    compare_qk(res, ref, torch.bfloat16, what="C3 ")
    del ref
    _sample_tokens_cpu_check(res, q, k, wq, wk, gq, gk, pos, inv, eps, torch.bfloat16)


# --------------------------------------------- Qwen3-8B packed sequences
def test_c4_qwen3_packed_bf16(cuda):
    eps = 1e-6
    gen = torch.Generator().manual_seed(300)
    pos = oracle.packed_position_ids(16, 8192, 64, 2048, gen).to(cuda)
    q, k, wq, wk, gq, gk = qk_inputs(16, 8192, 32, 8, 128, torch.bfloat16, cuda, seed=310)
    inv = oracle.inv_freq(128, 1e6).to(cuda)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv, eps)
    # check in two halves of the batch to bound the float64 working set
    for h in (slice(0, 8), slice(8, 16)):
        ref = oracle_qk(q[h], k[h], wq, wk, gq[h], gk[h], pos[h], inv, eps, device=cuda)
        for key in ("q_out", "k_out", "dq", "dk"):
            assert_tol(res[key][h], ref[key], torch.bfloat16, "C4 " + key)
        del ref
    for key, x, w, gg in (("dwq", q, wq, gq), ("dwk", k, wk, gk)):
        acc = torch.zeros(128, dtype=F64, device=cuda)
        for h in (slice(0, 8), slice(8, 16)):
            # float64 weight -> the oracle returns the unrounded float64 gradient
            r = oracle.qk_norm_rope_fwd_bwd(x[h], None, w.to(F64), None, gg[h], None, pos[h],
                                            inv, eps)
            acc += r["dwq"]
        assert_tol(res[key], acc, torch.bfloat16, "C4 " + key)
    _sample_tokens_cpu_check(res, q, k, wq, wk, gq, gk, pos, inv, eps, torch.bfloat16)


# ---------------------------------------------- sweep points with edge values
def _stress(shape, dtype, seed):
    """N(0,1) with 1% of elements x100 and ~0.1% (>=1) rows of zeros."""
    t = seeded_normal(shape, torch.float32, seed)
    flat = t.view(-1)
    gen = torch.Generator().manual_seed(seed + 1000)
    idx = torch.randperm(flat.numel(), generator=gen)[: flat.numel() // 100]
    flat[idx] *= 100
    rows = t.view(-1, shape[-1])
    nz = max(1, rows.shape[0] // 1000)
    rows[torch.randperm(rows.shape[0], generator=gen)[:nz]] = 0
    return t.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tokens", [2 ** 14])
def test_c5_sweep_point_with_outliers_and_zero_rows(cuda, dtype, tokens):
    eps = 1e-5
    x = _stress((tokens, 8192), dtype, 400).to(cuda)
    w = seeded_weight(8192, dtype, 401).to(cuda)
    g = seeded_normal((tokens, 8192), dtype, 402).to(cuda)
    y, dx, dw = run_rms(x, w, g, eps)
    ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x, w, g, eps)
    assert torch.isfinite(y).all() and torch.isfinite(dx).all()
    assert_tol(y, ry, dtype, "hidden y", True)
    # fp32 dx: bounded by the magnitude of the operands of its final difference,
    # rstd * (|dy*w| + |xhat*dot|), which rows of zeros scale by 1/sqrt(eps)
    assert_tol(dx, rdx, dtype, "hidden dx", True, oracle.rms_norm_dx_scale(x, w, g, eps))
    # fp32 dweight: bounded by the root-sum-square of its terms (1% of the
    # inputs are x100 outliers, so single columns can cancel to |dw| << terms)
    assert_tol(dw, rdw, dtype, "hidden dw", True, oracle.rms_norm_dw_scale(x, g, eps))
    del x, g, y, dx, ry, rdx

    q = _stress((1, tokens, 32, 128), dtype, 410).to(cuda)
    k = _stress((1, tokens, 8, 128), dtype, 411).to(cuda)
    wq = seeded_weight(128, dtype, 412).to(cuda)
    wk = seeded_weight(128, dtype, 413).to(cuda)
    gq = seeded_normal((1, tokens, 32, 128), dtype, 414).to(cuda)
    gk = seeded_normal((1, tokens, 8, 128), dtype, 415).to(cuda)
    inv = oracle.inv_freq(128, 5e5).to(cuda)
    res = run_qk(q, k, wq, wk, gq, gk, None, inv, eps)
    ref = oracle_qk(q, k, wq, wk, gq, gk, None, inv, eps, device=cuda)
    for key in ("q_out", "k_out"):
        assert_tol(res[key], ref[key], dtype, f"C5 {dtype} {key}", True)
    for key, x, w, gg in (("dq", q, wq, gq), ("dk", k, wk, gk)):
        assert_tol(res[key], ref[key], dtype, f"C5 {dtype} {key}", True,
                   oracle.qk_dx_scale(x, w, gg, None, inv, eps))
    for key, x, gg in (("dwq", q, gq), ("dwk", k, gk)):
        assert_tol(res[key], ref[key], dtype, f"C5 {dtype} {key}", True,
                   oracle.qk_dw_scale(x, gg, None, inv, eps))


# ------------------------------------------------------------------ edge cases
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_head_dims_and_dtypes(cuda, dtype, D):
    q, k, wq, wk, gq, gk = qk_inputs(2, 37, 5, 3, D, dtype, cuda, seed=D)
    inv = oracle.inv_freq(D, 1e4).to(cuda)
    pos = torch.randint(0, 5000, (2, 37), generator=torch.Generator().manual_seed(1)).to(cuda)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos, inv, 1e-6)
    compare_qk(res, ref, dtype, what=f"D{D} {dtype} ")


def test_qk_variants(cuda):
    dt = torch.bfloat16
    q, k, wq, wk, gq, gk = qk_inputs(3, 50, 4, 2, 128, dt, cuda, seed=500, wdtype=torch.float32)
    inv = oracle.inv_freq(128, 1e6).to(cuda)
    # int32 positions broadcast over the batch, fp32 weights with bf16 tensors
    pos = torch.arange(7, 57, dtype=torch.int32, device=cuda).view(1, 50)
    res = run_qk(q, k, wq, wk, gq, gk, pos, inv)
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos.long().expand(3, 50), inv)
    compare_qk(res, ref, dt, what="int32/bcast ")
    assert res["dwq"].dtype == torch.float32
    # q only
    res = run_qk(q, None, wq, None, gq, None, pos, inv)
    ref = oracle_qk(q, None, wq, None, gq, None, pos.long().expand(3, 50), inv)
    compare_qk(res, ref, dt, what="q only ")
    # strided q/k: slices of a packed [B, S, Hq+2Hk, D] projection output
    qkv = seeded_normal((3, 50, 8, 128), dt, 501).to(cuda)
    qs, ks = qkv[:, :, :4], qkv[:, :, 4:6]
    res = run_qk(qs, ks, wq, wk, gq, gk, pos, inv)
    ref = oracle_qk(qs, ks, wq, wk, gq, gk, pos.long().expand(3, 50), inv)
    compare_qk(res, ref, dt, what="strided ")
    # position-indexed bf16 table [P, D/2] and HF token-indexed [B, S, D] table
    ct, st = oracle.rope_cos_sin(torch.arange(200), inv.cpu(), torch.float32)
    res = run_qk(q, k, wq, wk, gq, gk, pos, None, cos=ct.bfloat16().to(cuda),
                 sin=st.bfloat16().to(cuda))
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos.long().expand(3, 50), None,
                    cos=ct.bfloat16(), sin=st.bfloat16())
    compare_qk(res, ref, dt, what="table ")
    emb_c = torch.cat([ct[7:57], ct[7:57]], -1).expand(3, 50, 128).contiguous()
    emb_s = torch.cat([st[7:57], st[7:57]], -1).expand(3, 50, 128).contiguous()
    res = run_qk(q, k, wq, wk, gq, gk, None, None, cos=emb_c.to(cuda), sin=emb_s.to(cuda))
    ref = oracle_qk(q, k, wq, wk, gq, gk, pos.long().expand(3, 50), None, cos=ct, sin=st)
    compare_qk(res, ref, dt, what="hf table ")


def test_rmsnorm_edge_shapes(cuda):
    for dtype in (torch.float32, torch.bfloat16):
        for M, N in ((1, 64), (3, 1000), (5, 4100), (17, 8), (2, 65536 if dtype != torch.float32 else 32768)):
            x = seeded_normal((M, N), dtype, M + N).to(cuda)
            w = seeded_weight(N, dtype, 1).to(cuda)
            g = seeded_normal((M, N), dtype, 2).to(cuda)
            y, dx, dw = run_rms(x, w, g, 1e-6)
            ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x.cpu(), w.cpu(), g.cpu(), 1e-6)
            assert_tol(y.cpu(), ry, dtype, f"y {M}x{N}")
            assert_tol(dx.cpu(), rdx, dtype, f"dx {M}x{N}")
            assert_tol(dw.cpu(), rdw, dtype, f"dw {M}x{N}", True)
    # misaligned base pointer (odd element offset) and a strided row view
    base = seeded_normal((9 * 512 + 1,), torch.bfloat16, 3).to(cuda)
    x = base[1:].view(9, 512)
    w = seeded_weight(512, torch.bfloat16, 4).to(cuda)
    ry, _ = oracle.rms_norm(x.cpu(), w.cpu(), 1e-6)
    assert_tol(bloth_b200.rms_norm(x, w).cpu(), ry, torch.bfloat16, "misaligned")
    wide = seeded_normal((6, 1024), torch.bfloat16, 5).to(cuda)
    xs = wide[:, :512]
    assert_tol(bloth_b200.rms_norm(xs, w).cpu(), oracle.rms_norm(xs.cpu(), w.cpu())[0],
               torch.bfloat16, "strided rows")


def test_rmsnorm_row_widths_sharing_a_kernel_in_any_order(cuda):
    # fp32 rows of 1024 and of 520 run the same pipelined kernel with different
    # shared-memory sizes; a wide call after a narrow one must still launch
    for N in (1024, 520, 1024, 700, 1024):
        x = seeded_normal((300, N), torch.float32, N).to(cuda)
        w = seeded_weight(N, torch.float32, 1).to(cuda)
        g = seeded_normal((300, N), torch.float32, 2).to(cuda)
        y, dx, dw = run_rms(x, w, g, 1e-6)
        ry, _, rdx, rdw = oracle.rms_norm_fwd_bwd(x.cpu(), w.cpu(), g.cpu(), 1e-6)
        assert_tol(y.cpu(), ry, torch.float32, f"y N={N}")
        assert_tol(dx.cpu(), rdx, torch.float32, f"dx N={N}")
        assert_tol(dw.cpu(), rdw, torch.float32, f"dw N={N}", True)


def test_rmsnorm_empty_and_determinism(cuda):
    x = torch.empty(0, 256, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    w = torch.ones(256, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = bloth_b200.rms_norm(x, w)
    y.backward(torch.empty_like(y))
    assert y.shape == (0, 256) and float(w.grad.abs().max()) == 0.0
    x = seeded_normal((4096, 2048), torch.bfloat16, 9).to(cuda)
    w = seeded_weight(2048, torch.bfloat16, 10).to(cuda)
    g = seeded_normal((4096, 2048), torch.bfloat16, 11).to(cuda)
    a = run_rms(x, w, g, 1e-5)
    b = run_rms(x, w, g, 1e-5)
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    q, k, wq, wk, gq, gk = qk_inputs(2, 1000, 32, 8, 128, torch.bfloat16, cuda, seed=12)
    inv = oracle.inv_freq(128, 5e5).to(cuda)
    r1 = run_qk(q, k, wq, wk, gq, gk, None, inv)
    r2 = run_qk(q, k, wq, wk, gq, gk, None, inv)
    for key in r1:
        assert torch.equal(r1[key], r2[key]), key


def test_table_variant_edge_cases(cuda):
    # rows wider than the rotated part, reference golden (bf16)
    g = load("fused_rest_bf16")
    xr = g["x"].to(cuda).requires_grad_(True)
    wr = g["w"].to(cuda).requires_grad_(True)
    y = bloth_b200.kernels.fused_norm_rope(xr, wr, g["cos"].to(cuda), g["sin"].to(cuda), g["eps"])
    assert_tol(y.cpu(), g["y"], torch.bfloat16, "rest fwd vs reference")
    y.backward(g["dy"].to(cuda))
    _, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(g["x"], g["w"], g["cos"], g["sin"], g["dy"],
                                                    g["eps"])
    assert_tol(xr.grad.cpu(), rdx, torch.bfloat16, "rest dx")
    assert_tol(wr.grad.cpu(), rdw, torch.bfloat16, "rest dw")
    # half not a multiple of the vector width (scalar rotation path), fp32
    M, N, h = 33, 128, 36
    x = seeded_normal((M, N), torch.float32, 20).to(cuda).requires_grad_(True)
    w = seeded_weight(N, torch.float32, 21).to(cuda).requires_grad_(True)
    ang = seeded_normal((M, h), torch.float32, 22)
    cos, sin = ang.cos(), ang.sin()
    dy = seeded_normal((M, N), torch.float32, 23)
    y = bloth_b200.kernels.fused_norm_rope(x, w, cos.to(cuda), sin.to(cuda), 1e-6)
    y.backward(dy.to(cuda))
    ry, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(x.detach().cpu(), w.detach().cpu(), cos,
                                                     sin, dy, 1e-6)
    assert_tol(y.cpu(), ry, torch.float32, "scalar rope y")
    assert_tol(x.grad.cpu(), rdx, torch.float32, "scalar rope dx")
    assert_tol(w.grad.cpu(), rdw, torch.float32, "scalar rope dw")
    # module wrapper
    mod = bloth_b200.BlothFusedNormQKV(N).to(cuda)
    assert mod(x.detach().view(3, 11, N), cos.to(cuda), sin.to(cuda)).shape == (3, 11, N)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [32, 64, 128, 256])
@pytest.mark.parametrize("parts", [2, 4])
def test_paired_table_rows_with_strided_inputs(cuda, dtype, N, parts):
    # Rows rotated in full (half = N/2) or on their first half (half = N/4,
    # the other half normalised only) with staged tables take the paired
    # layout (a thread holds a column and its rotation partner, and for
    # half = N/4 two vectors past the rotated part), 4-64 rows per block at
    # these widths. Strided x and dy rows are bulk-copied one row at a time,
    # and 1001 rows leave a partial last block. The weight is applied as w + 1.
    from bloth_b200.kernels.fused_norm_qkv_rope import norm_rope_backward, norm_rope_forward
    M, h, eps, off = 1001, N // parts, 1e-6, 1.0
    x = seeded_normal((M, N + 8), dtype, 40).to(cuda)[:, :N]
    dy = seeded_normal((M, N + 8), dtype, 41).to(cuda)[:, :N]
    w = (seeded_weight(N, torch.float32, 42) - 1.0).to(dtype).to(cuda)
    ang = seeded_normal((M, h), torch.float32, 43) * 3.0
    cs_dtype = torch.float32 if dtype == torch.float32 else dtype
    cos, sin = ang.cos().to(cs_dtype).to(cuda), ang.sin().to(cs_dtype).to(cuda)
    assert x.stride(0) == N + 8 and dy.stride(0) == N + 8
    y, rstd = norm_rope_forward(x, w, cos, sin, eps, off)
    dx, dw = norm_rope_backward(dy, x, w, cos, sin, rstd, off)
    xc, dyc, cc, sc = x.cpu(), dy.cpu(), cos.cpu(), sin.cpu()
    weff = w.cpu().to(F64) + off
    ry, _, rdx, rdw = oracle.norm_rope_table_fwd_bwd(xc, weff, cc, sc, dyc, eps)
    assert_tol(y.cpu(), ry, dtype, "paired y")
    assert_tol(dx.cpu(), rdx, dtype, "paired dx")
    assert_tol(dw.cpu(), rdw, dtype, "paired dw", True,
               oracle.norm_rope_table_dw_scale(xc, cc, sc, dyc, eps))
    assert bloth_b200._lib.load().bloth_device_fault(0) == 0


def test_rope_only_autograd(cuda):
    for dtype in (torch.float32, torch.bfloat16):
        x = seeded_normal((2, 40, 6, 128), dtype, 30).to(cuda).requires_grad_(True)
        dy = seeded_normal((2, 40, 6, 128), dtype, 31).to(cuda)
        inv = oracle.inv_freq(128, 1e4).to(cuda)
        pos = torch.arange(40, device=cuda).expand(2, 40) + 3
        y = bloth_b200.apply_rope(x, pos, inv)
        y.backward(dy)
        ry, rdx = oracle.rope_fwd_bwd(x.detach().cpu(), dy.cpu(), pos.cpu(), inv.cpu())
        assert_tol(y.cpu(), ry, dtype, "rope y")
        assert_tol(x.grad.cpu(), rdx, dtype, "rope dx")


def test_unsupported_head_dim_raises(cuda):
    q = torch.randn(1, 4, 2, 96, device=cuda)
    with pytest.raises(RuntimeError, match="size out of the supported range"):
        bloth_b200.fused_qk_norm_rope(q, None, torch.ones(96, device=cuda), None, None,
                                      oracle.inv_freq(96, 1e4).to(cuda))


def test_patched_hf_model_matches_unpatched(cuda):
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    cfg = transformers.Qwen3Config(vocab_size=128, hidden_size=128, intermediate_size=256,
                                   num_hidden_layers=2, num_attention_heads=4,
                                   num_key_value_heads=2, head_dim=32)
    ref = transformers.Qwen3ForCausalLM(cfg).to(cuda)
    pat = transformers.Qwen3ForCausalLM(cfg).to(cuda)
    pat.load_state_dict(ref.state_dict())
    bloth_b200.patch_model(pat, verbose=False)
    ids = torch.randint(0, 128, (2, 24), device=cuda)
    lr = ref(ids, labels=ids)
    lp = pat(ids, labels=ids)
    assert float((lr.logits - lp.logits).abs().max()) < 1e-4
    lr.loss.backward()
    lp.loss.backward()
    for (n, a), (_, b) in zip(ref.named_parameters(), pat.named_parameters()):
        assert float((a.grad - b.grad).abs().max()) < 1e-4, n
