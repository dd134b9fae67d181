"""GPU parity of the path's extensions on the HuggingFace side: the (1 + w)
weighting of Gemma-family norms (weight_offset), HF's attention_scaling
(rope_scale), RoPE of q and k in one launch, the drop-in for HF's
apply_rotary_pos_emb, and whole tiny models patched with
patch_model(..., patch_attention=True) against the same models unpatched.

Kernel outputs are compared with the oracle (float64 on the CPU) under the
path's tolerance: fp32 max abs 1e-5, bf16 abs 2e-2 or rel 1.6e-2. Whole
models in fp32 must match HF's own fp32 forward and gradients to 1e-4 (the
two differ only in fp32 rounding order). A bf16 model cannot match HF's bf16
path element for element, because HF rounds intermediate values to bf16
where the kernels round once; there the test asks that the patched bf16
logits be no further from the fp32 model's than HF's own bf16 logits are
(within 25%).
"""
import pytest
import torch

import bloth_b200
import oracle
from oracle.reference_path import seeded_normal, seeded_weight, tolerance_ok

pytestmark = pytest.mark.gpu


def assert_tol(got, ref, dtype, what, scale=False):
    ok, worst = tolerance_ok(got.detach().cpu(), ref, dtype, scale_with_magnitude=scale)
    assert ok, f"{what}: worst excess over tolerance {worst:.3e}"


# ------------------------------------------------------- weight offset (Gemma)
@pytest.mark.parametrize("dtype,N", [(torch.float32, 1024), (torch.bfloat16, 4096),
                                     (torch.bfloat16, 1000)])
def test_rms_norm_weight_offset(cuda, dtype, N):
    M = 777
    x = seeded_normal((M, N), dtype, 1)
    w = (0.1 * seeded_normal((N,), torch.float32, 2)).to(dtype)  # Gemma: w near 0
    dy = seeded_normal((M, N), dtype, 3)
    ref_y, ref_r, ref_dx, ref_dw = oracle.rms_norm_fwd_bwd(x, w, dy, 1e-6, w_offset=1.0)
    xg = x.to(cuda).requires_grad_(True)
    wg = w.to(cuda).requires_grad_(True)
    y = bloth_b200.rms_norm(xg, wg, 1e-6, weight_offset=1.0)
    y.backward(dy.to(cuda))
    assert_tol(y, ref_y, dtype, "y")
    assert_tol(xg.grad, ref_dx, dtype, "dx")
    assert_tol(wg.grad, ref_dw, dtype, "dw", scale=True)


def test_offset_module_matches_hf_gemma_norm(cuda):
    transformers = pytest.importorskip("transformers")
    from transformers.models.gemma.modeling_gemma import GemmaRMSNorm
    hf = GemmaRMSNorm(512, eps=1e-6).to(cuda)
    with torch.no_grad():
        hf.weight.normal_(0.0, 0.1)
    ours = bloth_b200.BlothRMSNorm(512, 1e-6, weight_offset=1.0).to(cuda)
    ours.weight = hf.weight
    x = seeded_normal((64, 512), torch.float32, 5).to(cuda)
    with torch.no_grad():
        assert float((hf(x) - ours(x)).abs().max()) < 1e-5
    del transformers


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tables", [False, True])
def test_qk_weight_offset_and_rope_scale(cuda, dtype, tables):
    B, S, Hq, Hk, D = 2, 96, 4, 2, 128
    q = seeded_normal((B, S, Hq, D), dtype, 10)
    k = seeded_normal((B, S, Hk, D), dtype, 11)
    wq = (0.1 * seeded_normal((D,), torch.float32, 12)).to(dtype)
    wk = (0.1 * seeded_normal((D,), torch.float32, 13)).to(dtype)
    gq = seeded_normal((B, S, Hq, D), dtype, 14)
    gk = seeded_normal((B, S, Hk, D), dtype, 15)
    pos = torch.arange(S).unsqueeze(0).expand(B, S) + 7
    inv = oracle.inv_freq(D, 1e4)
    cos = sin = None
    if tables:
        c, s = oracle.rope_cos_sin(torch.arange(S + 7), inv, torch.float32)
        cos, sin, inv_use = c, s, None
    else:
        inv_use = inv
    scale = 0.8
    ref = oracle.qk_norm_rope_fwd_bwd(q, k, wq, wk, gq, gk, pos, inv_use, 1e-6, cos, sin,
                                      w_offset=1.0, rope_scale=scale)
    t = lambda x: None if x is None else x.to(cuda)  # noqa: E731
    qg, kg = t(q).requires_grad_(True), t(k).requires_grad_(True)
    wqg, wkg = t(wq).requires_grad_(True), t(wk).requires_grad_(True)
    qo, ko = bloth_b200.fused_qk_norm_rope(qg, kg, wqg, wkg, t(pos), t(inv_use), 1e-6,
                                           cos=t(cos), sin=t(sin), weight_offset=1.0,
                                           rope_scale=scale)
    torch.autograd.backward((qo, ko), (t(gq), t(gk)))
    for name, got in (("q_out", qo), ("k_out", ko), ("dq", qg.grad), ("dk", kg.grad)):
        assert_tol(got, ref[name], dtype, name)
    assert_tol(wqg.grad, ref["dwq"], dtype, "dwq", scale=True)
    assert_tol(wkg.grad, ref["dwk"], dtype, "dwk", scale=True)


# ------------------------------------------------------------ RoPE of q and k
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_qk_one_launch(cuda, dtype):
    B, S, Hq, Hk, D = 2, 80, 8, 2, 64
    q = seeded_normal((B, S, Hq, D), dtype, 20)
    k = seeded_normal((B, S, Hk, D), dtype, 21)
    gq = seeded_normal((B, S, Hq, D), dtype, 22)
    gk = seeded_normal((B, S, Hk, D), dtype, 23)
    pos = torch.randint(0, 4000, (B, S), generator=torch.Generator().manual_seed(24))
    inv = oracle.inv_freq(D, 5e5)
    yq, dq = oracle.rope_fwd_bwd(q, gq, pos, inv, rope_scale=1.25)
    yk, dk = oracle.rope_fwd_bwd(k, gk, pos, inv, rope_scale=1.25)
    qg = q.to(cuda).requires_grad_(True)
    kg = k.to(cuda).requires_grad_(True)
    qo, ko = bloth_b200.apply_rope_qk(qg, kg, pos.to(cuda), inv.to(cuda), rope_scale=1.25)
    torch.autograd.backward((qo, ko), (gq.to(cuda), gk.to(cuda)))
    assert_tol(qo, yq, dtype, "q_out")
    assert_tol(ko, yk, dtype, "k_out")
    assert_tol(qg.grad, dq, dtype, "dq")
    assert_tol(kg.grad, dk, dtype, "dk")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_apply_rotary_pos_emb_matches_hf(cuda, dtype):
    transformers = pytest.importorskip("transformers")
    from transformers.models.llama import modeling_llama as ml
    cfg = transformers.LlamaConfig(hidden_size=512, num_attention_heads=4, head_dim=128,
                                   rope_theta=5e5)
    rot = ml.LlamaRotaryEmbedding(cfg).to(cuda)
    B, S = 2, 64
    x = seeded_normal((B, S, 512), dtype, 30).to(cuda)
    pos = torch.arange(S, device=cuda).unsqueeze(0).expand(B, S)
    cos, sin = rot(x, pos)
    q = seeded_normal((B, S, 4, 128), dtype, 31).to(cuda).transpose(1, 2)
    k = seeded_normal((B, S, 2, 128), dtype, 32).to(cuda).transpose(1, 2)
    ref = [t.float() for t in ml.apply_rotary_pos_emb(q.float(), k.float(), cos.float(),
                                                       sin.float())]
    got = bloth_b200.apply_rotary_pos_emb(q, k, cos, sin)
    assert got[0].shape == q.shape and got[1].shape == k.shape
    for g, r, what in zip(got, ref, ("q", "k")):
        assert_tol(g, r.double().cpu(), dtype, what)


# ------------------------------------------------------------ whole models
def _tiny(kind, dtype, dev, seed=0, **extra):
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(seed)
    common = dict(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, **extra)
    if kind == "qwen3":
        cfg = transformers.Qwen3Config(head_dim=64, **common)
        cls = transformers.Qwen3ForCausalLM
    elif kind == "llama":
        cfg = transformers.LlamaConfig(head_dim=64, **common)
        cls = transformers.LlamaForCausalLM
    elif kind == "mistral":
        cfg = transformers.MistralConfig(head_dim=64, **common)
        cls = transformers.MistralForCausalLM
    elif kind == "qwen2":
        cfg = transformers.Qwen2Config(**common)
        cls = transformers.Qwen2ForCausalLM
    elif kind == "gemma":
        cfg = transformers.GemmaConfig(head_dim=64, **common)
        cls = transformers.GemmaForCausalLM
    else:
        raise ValueError(kind)
    cfg._attn_implementation = "eager"
    ref = cls(cfg).to(dev)
    if kind == "gemma":  # zero-initialised (1 + w) weights: make them non-trivial
        with torch.no_grad():
            for n, p in ref.named_parameters():
                if "norm" in n:
                    p.normal_(0.0, 0.1)
    ref = ref.to(dtype)
    pat = cls(cfg).to(dev).to(dtype)
    pat.load_state_dict(ref.state_dict())
    return ref, pat


@pytest.mark.parametrize("kind", ["qwen3", "llama", "mistral", "qwen2", "gemma"])
def test_patched_model_fp32_matches_hf(cuda, kind):
    ref, pat = _tiny(kind, torch.float32, cuda)
    bloth_b200.patch_model(pat, patch_attention=True, verbose=False)
    if kind != "gemma":
        assert all(getattr(m, "_bloth_attention", None) is not None
                   for m in pat.modules() if type(m).__name__.endswith("Attention"))
    ids = torch.randint(0, 128, (2, 48), device=cuda,
                        generator=torch.Generator(device=cuda).manual_seed(1))
    lr = ref(ids, labels=ids)
    lp = pat(ids, labels=ids)
    assert float((lr.logits - lp.logits).detach().abs().max()) < 1e-4
    lr.loss.backward()
    lp.loss.backward()
    for (n, a), (_, b) in zip(ref.named_parameters(), pat.named_parameters()):
        assert float((a.grad - b.grad).abs().max()) < 1e-4, n


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_patched_model_bf16_no_worse_than_hf_bf16(cuda, kind):
    ref32, _ = _tiny(kind, torch.float32, cuda)
    hf16, pat16 = _tiny(kind, torch.bfloat16, cuda)
    bloth_b200.patch_model(pat16, patch_attention=True, verbose=False)
    ids = torch.randint(0, 128, (2, 48), device=cuda,
                        generator=torch.Generator(device=cuda).manual_seed(2))
    with torch.no_grad():
        truth = ref32(ids).logits
        err_hf = float((hf16(ids).logits.float() - truth).abs().max())
        err_pat = float((pat16(ids).logits.float() - truth).abs().max())
    assert err_pat <= 1.25 * err_hf + 1e-3, (err_pat, err_hf)


def test_patched_model_generates_with_kv_cache(cuda):
    ref, pat = _tiny("qwen3", torch.float32, cuda)
    bloth_b200.patch_model(pat, patch_attention=True, verbose=False)
    ids = torch.randint(0, 128, (1, 12), device=cuda,
                        generator=torch.Generator(device=cuda).manual_seed(3))
    a = ref.generate(ids, max_new_tokens=8, do_sample=False)
    b = pat.generate(ids, max_new_tokens=8, do_sample=False)
    assert torch.equal(a, b)


# ------------------------------------------------------ residual add + RMSNorm
@pytest.mark.parametrize("dtype,M,N", [(torch.bfloat16, 333, 4096), (torch.float32, 300, 1024),
                                       (torch.bfloat16, 97, 4100), (torch.bfloat16, 8, 65536),
                                       (torch.float32, 8, 32768), (torch.float16, 64, 2048)])
@pytest.mark.parametrize("with_dz", [True, False])
def test_fused_add_rms_norm(cuda, dtype, M, N, with_dz):
    x = seeded_normal((M, N), dtype, 40)
    r = seeded_normal((M, N), dtype, 41)
    w = seeded_weight(N, dtype, 42)
    dy = seeded_normal((M, N), dtype, 43)
    dz = seeded_normal((M, N), dtype, 44) if with_dz else None
    ry, rz, _, rdx, rdw = oracle.add_rms_norm_fwd_bwd(x, r, w, dy, dz, 1e-6)
    xg = x.to(cuda).requires_grad_(True)
    rg = r.to(cuda).requires_grad_(True)
    wg = w.to(cuda).requires_grad_(True)
    y, z = bloth_b200.fused_add_rms_norm(xg, rg, wg, 1e-6)
    outs, grads = [y], [dy.to(cuda)]
    if with_dz:
        outs.append(z)
        grads.append(dz.to(cuda))
    torch.autograd.backward(outs, grads)
    assert torch.equal(z.cpu(), rz), "z = x + r must round exactly as the dtype's add"
    assert_tol(y, ry, dtype, "y")
    assert_tol(xg.grad, rdx, dtype, "dx")
    assert_tol(rg.grad, rdx, dtype, "dr")
    assert_tol(wg.grad, rdw, dtype, "dw", scale=True)


def test_fused_add_rms_norm_in_place_through_the_abi(cuda):
    from bloth_b200 import _lib
    M, N = 500, 4096
    x = seeded_normal((M, N), torch.bfloat16, 50)
    r = seeded_normal((M, N), torch.bfloat16, 51)
    w = seeded_weight(N, torch.bfloat16, 52)
    ry, rz, rrs, _, _ = oracle.add_rms_norm_fwd_bwd(x, r, w, torch.zeros_like(x), None, 1e-5)
    xd, rd, wd = x.to(cuda), r.to(cuda), w.to(cuda)
    y = torch.empty_like(xd)
    rstd = torch.empty(M, dtype=torch.float32, device=cuda)
    lib = _lib.load()
    rc = lib.bloth_add_rmsnorm_fwd(_lib.ptr(xd), N, _lib.ptr(rd), N, _lib.ptr(rd), N,
                                   _lib.ptr(wd), 0.0, _lib.ptr(y), N, _lib.ptr(rstd), M, N, 1e-5,
                                   _lib.BF16, _lib.BF16, _lib.stream_of(xd))
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.equal(rd.cpu(), rz)  # the residual buffer now holds z
    assert_tol(y, ry, torch.bfloat16, "y")
    assert_tol(rstd, rrs, torch.float32, "rstd")


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_patched_residual_model_fp32_matches_hf(cuda, kind):
    ref, pat = _tiny(kind, torch.float32, cuda)
    bloth_b200.patch_model(pat, patch_attention=True, patch_residual=True, verbose=False)
    ids = torch.randint(0, 128, (2, 48), device=cuda,
                        generator=torch.Generator(device=cuda).manual_seed(4))
    lr = ref(ids, labels=ids)
    lp = pat(ids, labels=ids)
    assert float((lr.logits - lp.logits).detach().abs().max()) < 1e-4
    lr.loss.backward()
    lp.loss.backward()
    for (n, a), (_, b) in zip(ref.named_parameters(), pat.named_parameters()):
        assert float((a.grad - b.grad).abs().max()) < 1e-4, n


ROPE_PARAMS = {
    "yarn": {"rope_type": "yarn", "factor": 4.0, "rope_theta": 1e4,
             "original_max_position_embeddings": 32},
    "llama3": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
               "high_freq_factor": 4.0, "original_max_position_embeddings": 32,
               "rope_theta": 5e5},
    "linear": {"rope_type": "linear", "factor": 2.0, "rope_theta": 1e4},
}


def _compare(ref, pat, dev, seq=48, mask=None, grads=True, tol=1e-4):
    ids = torch.randint(0, 128, (2, seq), device=dev,
                        generator=torch.Generator(device=dev).manual_seed(7))
    kw = {} if mask is None else {"attention_mask": mask}
    lr = ref(ids, labels=ids, **kw)
    lp = pat(ids, labels=ids, **kw)
    keep = slice(None) if mask is None else mask.bool()
    assert float((lr.logits[keep] - lp.logits[keep]).detach().abs().max()) < tol
    if grads:
        lr.loss.backward()
        lp.loss.backward()
        for (n, a), (_, b) in zip(ref.named_parameters(), pat.named_parameters()):
            assert float((a.grad - b.grad).abs().max()) < tol, n


@pytest.mark.parametrize("rope", sorted(ROPE_PARAMS))
@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_patched_model_with_scaled_rope(cuda, kind, rope):
    # HF's rotary embedding folds the rope type (and YaRN's attention_scaling
    # != 1) into its cos/sin tables, which the binding reads as they are
    ref, pat = _tiny(kind, torch.float32, cuda, rope_parameters=dict(ROPE_PARAMS[rope]))
    bloth_b200.patch_model(pat, patch_attention=True, patch_residual=True, verbose=False)
    _compare(ref, pat, cuda)


def test_in_register_rope_scale_matches_hf_yarn_tables(cuda):
    transformers = pytest.importorskip("transformers")
    from transformers.models.llama import modeling_llama as ml
    cfg = transformers.LlamaConfig(hidden_size=512, num_attention_heads=4, head_dim=128,
                                   rope_parameters=dict(ROPE_PARAMS["yarn"]))
    rot = ml.LlamaRotaryEmbedding(cfg).to(cuda)
    assert abs(rot.attention_scaling - 1.0) > 0.1
    B, S = 2, 200
    pos = torch.arange(S, device=cuda).unsqueeze(0).expand(B, S)
    cos, sin = rot(torch.zeros(1, device=cuda), pos)  # fp32 tables, scaling included
    q = seeded_normal((B, S, 4, 128), torch.float32, 60).to(cuda)
    k = seeded_normal((B, S, 2, 128), torch.float32, 61).to(cuda)
    wq = seeded_weight(128, torch.float32, 62).to(cuda)
    wk = seeded_weight(128, torch.float32, 63).to(cuda)
    a = bloth_b200.fused_qk_norm_rope(q, k, wq, wk, pos, rot.inv_freq.float(), 1e-6,
                                      rope_scale=rot.attention_scaling)
    b = bloth_b200.fused_qk_norm_rope(q, k, wq, wk, None, None, 1e-6, cos=cos, sin=sin)
    for x, y in zip(a, b):
        assert float((x - y).abs().max()) < 1e-5


def test_patched_mistral_sliding_window(cuda):
    ref, pat = _tiny("mistral", torch.float32, cuda, sliding_window=16)
    bloth_b200.patch_model(pat, patch_attention=True, patch_residual=True, verbose=False)
    _compare(ref, pat, cuda, seq=48)


def test_patched_model_left_padding(cuda):
    ref, pat = _tiny("llama", torch.float32, cuda)
    bloth_b200.patch_model(pat, patch_attention=True, patch_residual=True, verbose=False)
    mask = torch.ones(2, 40, dtype=torch.long, device=cuda)
    mask[0, :7] = 0  # left padding in the first sequence
    with torch.no_grad():
        _compare(ref, pat, cuda, seq=40, mask=mask, grads=False)


def test_patched_model_fp16_no_worse_than_hf_fp16(cuda):
    ref32, _ = _tiny("llama", torch.float32, cuda)
    hf16, pat16 = _tiny("llama", torch.float16, cuda)
    bloth_b200.patch_model(pat16, patch_attention=True, patch_residual=True, verbose=False)
    ids = torch.randint(0, 128, (2, 48), device=cuda,
                        generator=torch.Generator(device=cuda).manual_seed(8))
    with torch.no_grad():
        truth = ref32(ids).logits
        err_hf = float((hf16(ids).logits.float() - truth).abs().max())
        err_pat = float((pat16(ids).logits.float() - truth).abs().max())
    assert err_pat <= 1.25 * err_hf + 1e-3, (err_pat, err_hf)
