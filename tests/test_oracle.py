"""Pins the CPU oracle against golden vectors produced by the reference's own
Triton kernels (tests/golden/make_golden.py), and checks its internal
consistency. CPU only."""
import pytest
import torch

import oracle
from oracle.reference_path import tolerance_ok
from tests.golden import load


def _close(a, b, atol):
    return float((a.to(torch.float64) - b.to(torch.float64)).abs().max()) <= atol


def test_rmsnorm_f32_matches_reference_fwd_bwd():
    g = load("rmsnorm_f32")
    y, rstd, dx, dw = oracle.rms_norm_fwd_bwd(g["x"], g["w"], g["dy"], g["eps"])
    assert _close(y, g["y"], 1e-5)
    assert _close(rstd, g["rstd"], 1e-5)
    assert _close(dx, g["dx"], 1e-5)
    assert _close(dw, g["dw"], 1e-4)  # reference sums 64 fp32 atomics in arbitrary order


def _bf16_truncate(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by dropping the low 16 bits (round toward zero), which is
    how Triton's CPU interpreter stores bf16; GPU Triton and torch round to
    nearest even."""
    bits = t.to(torch.float32).contiguous().view(torch.int32) & ~0xFFFF
    return bits.view(torch.float32).to(torch.bfloat16)


def test_rmsnorm_bf16_matches_reference_test_golden():
    # the reference's own test case: bf16 x, unit weight, M=256, N=2048
    # (bloth/tests/test_kernels.py:119-134)
    g = load("rmsnorm_bf16")
    y, _ = oracle.rms_norm(g["x"], g["w"], g["eps"])
    assert y.dtype == torch.bfloat16
    # within the path's bf16 tolerance of the interpreter-run reference
    ok, worst = tolerance_ok(y, g["y"], torch.bfloat16)
    assert ok, worst
    # bit-exact once the interpreter's truncating bf16 store is applied to the
    # oracle's fp32-computed value
    ref_like = _bf16_truncate(oracle.rms_norm(g["x"].float(), g["w"].float(), g["eps"],
                                              compute=torch.float32)[0])
    assert (ref_like.view(torch.int16) == g["y"].view(torch.int16)).float().mean() > 0.999
    # and the oracle's round-to-nearest result is within one bf16 ulp everywhere
    ulp = torch.finfo(torch.bfloat16).eps * g["y"].float().abs().clamp(min=2**-126)
    assert bool(((y.float() - g["y"].float()).abs() <= 2 * ulp).all())


def _row_tables(g, H):
    S = g["cos"].shape[0]
    pos = torch.arange(S).view(1, S, 1).expand(2, S, H).reshape(-1)
    return g["cos"][pos], g["sin"][pos]


def test_fused_fwd_matches_reference_q_k():
    for name, H in (("q", 8), ("k", 2)):
        g = load(f"fused_{name}_f32")
        D = g["x"].shape[-1]
        cos, sin = _row_tables(g, H)
        y, rstd = oracle.norm_rope_table(g["x"].view(-1, D), g["w"], cos, sin, g["eps"])
        assert _close(y.view_as(g["x"]), g["y"], 1e-5), name
        assert _close(rstd, g["rstd"], 1e-5), name


def test_position_form_equals_table_form():
    # the in-register cos/sin form (positions + inv_freq) reproduces the
    # reference's fp32 table form on the CPU correctness config
    g = load("fused_q_f32")
    B, S, H, D = g["x"].shape
    inv = oracle.inv_freq(D, g["theta"])
    q_out, _, rq, _ = oracle.qk_norm_rope(g["x"], None, g["w"], None, None, inv, g["eps"])
    assert _close(q_out, g["y"], 1e-5)
    assert _close(rq.reshape(-1), g["rstd"], 1e-5)


def test_reference_fused_backward_is_plain_rmsnorm_backward():
    # The reference's fused backward kernel (fused_norm_qkv_rope.py:99-126)
    # leaves out the transposed rotation: it equals the RMSNorm backward of dy,
    # not the gradient of the fused forward.
    for name in ("fused_k_f32", "fused_rest_bf16"):
        g = load(name)
        x = g["x"].reshape(-1, g["x"].shape[-1])
        dy = g["dy"].reshape_as(x)
        dx_ref, dw_ref = oracle.norm_rope_table_reference_bwd(x, g["w"], g["rstd"], dy)
        ok, worst = tolerance_ok(dx_ref, g["ref_bwd_dx"].reshape_as(x), x.dtype)
        assert ok, (name, worst)
        if x.dtype == torch.float32:
            # the reference sums dw with M fp32 atomics, a few ulps from the exact sum
            assert _close(dw_ref, g["ref_bwd_dw"], 1e-4 * max(1.0, float(dw_ref.abs().max())))
        else:
            ok, worst = tolerance_ok(dw_ref, g["ref_bwd_dw"], x.dtype)
            assert ok, (name, worst)
    # ... and differs from the exact gradient by O(1)
    g = load("fused_k_f32")
    B, S, H, D = g["x"].shape
    cos, sin = _row_tables(g, H)
    x = g["x"].view(-1, D)
    _, _, dx, _ = oracle.norm_rope_table_fwd_bwd(x, g["w"], cos, sin, g["dy"].view(-1, D),
                                                 g["eps"])
    assert float((dx - g["ref_bwd_dx"].view(-1, D)).abs().max()) > 0.5


def test_fused_rest_columns_bf16():
    g = load("fused_rest_bf16")
    y, rstd = oracle.norm_rope_table(g["x"], g["w"], g["cos"], g["sin"], g["eps"])
    ok, worst = tolerance_ok(y, g["y"], torch.bfloat16)
    assert ok, worst
    assert _close(rstd, g["rstd"], 1e-5)


def test_rope_embedding_matches_reference_bf16():
    g = load("rope_bf16")
    x = g["x"]  # [b, h, s, d]
    y = oracle.rope(x.transpose(1, 2), cos=g["cos"], sin=g["sin"]).transpose(1, 2)
    ok, worst = tolerance_ok(y, g["y"], torch.bfloat16)
    assert ok, worst


def test_oracle_gradients_are_exact():
    torch.manual_seed(0)
    x = torch.randn(3, 5, 2, 8, dtype=torch.float64, requires_grad=True)
    w = (1 + 0.1 * torch.randn(8, dtype=torch.float64)).requires_grad_()
    inv = oracle.inv_freq(8, 1e4)

    def f(x_, w_):
        q, _, _, _ = oracle.qk_norm_rope(x_, None, w_, None, None, inv, 1e-6)
        return q

    assert torch.autograd.gradcheck(f, (x, w))


def test_packed_position_ids_properties():
    g = torch.Generator().manual_seed(0)
    p = oracle.packed_position_ids(4, 8192, 64, 2048, g)
    assert p.shape == (4, 8192)
    for r in range(4):
        starts = (p[r] == 0).nonzero().flatten().tolist() + [8192]
        lens = [b - a for a, b in zip(starts[:-1], starts[1:])]
        assert sum(lens) == 8192
        assert all(64 <= n <= 2048 for n in lens)
        for a, n in zip(starts[:-1], lens):
            assert torch.equal(p[r, a:a + n], torch.arange(n))


def test_gemma_norm_is_the_unit_offset_not_the_references_replacement():
    # transformers' GemmaRMSNorm computes x_hat * (1 + w); the reference's
    # patcher (bloth/bloth/patch.py:33-34 with :46-76) puts an x_hat * w norm
    # in its place, which for Gemma's zero-initialised weights outputs zeros
    transformers = pytest.importorskip("transformers")
    from transformers.models.gemma.modeling_gemma import GemmaRMSNorm
    g = torch.Generator().manual_seed(3)
    x = torch.randn(16, 256, generator=g)
    hf = GemmaRMSNorm(256, eps=1e-6)
    with torch.no_grad():
        hf.weight.normal_(0.0, 0.1, generator=g)
        want = hf(x)
    w = hf.weight.detach()
    ours, _ = oracle.rms_norm(x, w, 1e-6, compute=torch.float32, w_offset=1.0)
    assert torch.allclose(ours, want, atol=1e-6)
    as_reference_patches_it, _ = oracle.rms_norm(x, w, 1e-6, compute=torch.float32)
    assert float((as_reference_patches_it - want).abs().max()) > 0.5
    fresh = GemmaRMSNorm(256, eps=1e-6)
    with torch.no_grad():
        assert float(oracle.rms_norm(x, fresh.weight, 1e-6)[0].abs().max()) == 0.0
        assert float(fresh(x).abs().max()) > 1.0
