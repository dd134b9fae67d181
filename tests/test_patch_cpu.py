"""The HuggingFace patcher on CPU: which modules it replaces or binds, with
which parameters. No kernel runs here (forward passes are GPU tests)."""
import warnings

import pytest
import torch

import bloth_b200
from bloth_b200.attention import _ATTENTION_CLASSES, _attention_forward

transformers = pytest.importorskip("transformers")


def _tiny(kind: str, head_dim: int = 64, **extra):
    common = dict(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=2, num_key_value_heads=1, **extra)
    if kind == "qwen3":
        return transformers.Qwen3ForCausalLM(transformers.Qwen3Config(head_dim=head_dim, **common))
    if kind == "llama":
        return transformers.LlamaForCausalLM(transformers.LlamaConfig(head_dim=head_dim, **common))
    if kind == "mistral":
        return transformers.MistralForCausalLM(
            transformers.MistralConfig(head_dim=head_dim, **common))
    if kind == "qwen2":
        common = dict(common, hidden_size=2 * head_dim)
        return transformers.Qwen2ForCausalLM(transformers.Qwen2Config(**common))
    if kind == "gemma":
        return transformers.GemmaForCausalLM(transformers.GemmaConfig(head_dim=head_dim, **common))
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["qwen3", "llama", "mistral", "qwen2"])
def test_patch_attention_binds_every_layer(kind):
    model = _tiny(kind)
    keys = set(model.state_dict())
    bloth_b200.patch_model(model, patch_attention=True, verbose=False)
    attn = [m for m in model.modules() if type(m).__name__ in _ATTENTION_CLASSES]
    assert len(attn) == 2
    for m in attn:
        assert m.forward.__func__ is _attention_forward
        assert m._bloth_attention.norms == (kind == "qwen3")
    assert set(model.state_dict()) == keys
    # a second call binds nothing more
    assert bloth_b200.attention.patch_attention_layers(model, verbose=False) == 0


def test_patch_attention_is_per_instance():
    a, b = _tiny("llama"), _tiny("llama")
    bloth_b200.patch_model(a, patch_attention=True, verbose=False)
    for m in b.modules():
        if type(m).__name__ == "LlamaAttention":
            assert "forward" not in m.__dict__


def test_patch_attention_skips_unsupported_head_dim():
    model = _tiny("qwen3", head_dim=32)
    with warnings.catch_warnings(record=True) as rec:
        warnings.simplefilter("always")
        n = bloth_b200.attention.patch_attention_layers(model, verbose=False)
    assert n == 0
    assert any("head_dim 32" in str(w.message) for w in rec)


def test_patch_attention_false_leaves_attention_alone():
    model = _tiny("qwen3")
    bloth_b200.patch_model(model, verbose=False)
    for m in model.modules():
        assert "forward" not in m.__dict__


def test_gemma_norms_get_the_unit_offset():
    model = _tiny("gemma")
    before = {n: m.weight for n, m in model.named_modules()
              if type(m).__name__ == "GemmaRMSNorm"}
    bloth_b200.patch_model(model, verbose=False)
    after = {n: m for n, m in model.named_modules() if type(m).__name__ == "BlothRMSNorm"}
    assert len(after) == len(before) == 5
    for n, m in after.items():
        assert m.weight is before[n]
        assert m.weight_offset == 1.0


def test_fresh_offset_norm_is_identity_scale():
    norm = bloth_b200.BlothRMSNorm(8, weight_offset=1.0)
    assert torch.equal(norm.weight.detach(), torch.zeros(8))
    assert torch.equal(bloth_b200.BlothRMSNorm(8).weight.detach(), torch.ones(8))


def test_layernorm_on_the_reference_list_is_left_in_place():
    class CohereLayerNorm(torch.nn.Module):  # same class name as transformers'
        def __init__(self):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.ones(16))
            self.variance_epsilon = 1e-5

    model = torch.nn.Sequential(CohereLayerNorm())
    assert bloth_b200.patch.patch_model(model, verbose=False) is model
    assert type(model[0]).__name__ == "CohereLayerNorm"


def _oracle_kernels(monkeypatch):
    """Stands the oracle in for the two kernels the binding calls, so the
    binding's host logic (layouts, cache update, attention call) runs on CPU."""
    import oracle
    from bloth_b200 import attention

    def qk(q, k, wq, wk, eps=1e-6, cos=None, sin=None, weight_offset=0.0):
        qo, ko, _, _ = oracle.qk_norm_rope(q, k, wq, wk, None, None, eps, cos, sin,
                                           compute=torch.float32, w_offset=weight_offset)
        return qo, ko

    def rope_qk(q, k, cos=None, sin=None):
        return (oracle.rope(q, cos=cos, sin=sin, compute=torch.float32),
                oracle.rope(k, cos=cos, sin=sin, compute=torch.float32))

    monkeypatch.setattr(attention, "fused_qk_norm_rope", qk)
    monkeypatch.setattr(attention, "apply_rope_qk", rope_qk)


@pytest.mark.parametrize("kind", ["qwen3", "llama", "mistral", "qwen2"])
def test_attention_binding_host_logic(monkeypatch, kind):
    _oracle_kernels(monkeypatch)
    torch.manual_seed(0)
    ref = _tiny(kind)
    pat = _tiny(kind)
    pat.load_state_dict(ref.state_dict())
    bloth_b200.patch_model(pat, patch_norms=False, patch_attention=True, verbose=False)
    ids = torch.randint(0, 64, (2, 20), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        a, b = ref(ids).logits, pat(ids).logits
    assert float((a - b).abs().max()) < 1e-4
    if kind == "qwen3":  # incremental decoding through the KV cache
        ga = ref.generate(ids[:1], max_new_tokens=6, do_sample=False)
        gb = pat.generate(ids[:1], max_new_tokens=6, do_sample=False)
        assert torch.equal(ga, gb)


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_residual_binding_host_logic(monkeypatch, kind):
    import oracle
    from bloth_b200 import attention

    def add_norm(x, r, w, eps=1e-6, weight_offset=0.0):
        z = x + r
        return oracle.rms_norm(z, w, eps, compute=torch.float32, w_offset=weight_offset)[0], z

    monkeypatch.setattr(attention, "fused_add_rms_norm", add_norm)
    _oracle_kernels(monkeypatch)
    torch.manual_seed(0)
    ref, pat = _tiny(kind), _tiny(kind)
    pat.load_state_dict(ref.state_dict())
    bloth_b200.patch_model(pat, patch_norms=False, patch_attention=True, patch_residual=True,
                           verbose=False)
    layers = [m for m in pat.modules() if type(m).__name__.endswith("DecoderLayer")]
    assert len(layers) == 2 and all("forward" in m.__dict__ for m in layers)
    ids = torch.randint(0, 64, (2, 20), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        a, b = ref(ids).logits, pat(ids).logits
    assert float((a - b).abs().max()) < 1e-4
    # a second call binds nothing more
    assert attention.patch_decoder_layers(pat, verbose=False) == 0


def test_add_rms_norm_oracle_gradients():
    import oracle
    g = torch.Generator().manual_seed(5)
    x, r, dy, dz = (torch.randn(6, 32, generator=g, dtype=torch.float64) for _ in range(4))
    w = torch.randn(32, generator=g, dtype=torch.float64)
    y, z, _, dx, dw = oracle.add_rms_norm_fwd_bwd(x, r, w, dy, dz, 1e-6)
    # against autograd of the unfused ops
    xa, ra, wa = (t.clone().requires_grad_(True) for t in (x, r, w))
    za = xa + ra
    ya = za * torch.rsqrt((za * za).mean(-1, keepdim=True) + 1e-6) * wa
    torch.autograd.backward([ya, za], [dy, dz])
    assert torch.allclose(y, ya) and torch.allclose(z, za)
    assert torch.allclose(dx, xa.grad) and torch.allclose(dx, ra.grad)
    assert torch.allclose(dw, wa.grad)


@pytest.mark.parametrize("kind,extra", [
    ("llama", {"rope_parameters": {"rope_type": "yarn", "factor": 4.0, "rope_theta": 1e4,
                                   "original_max_position_embeddings": 32}}),
    ("qwen3", {"rope_parameters": {"rope_type": "linear", "factor": 2.0, "rope_theta": 1e4}}),
    ("mistral", {"sliding_window": 8}),
])
def test_attention_binding_host_logic_variants(monkeypatch, kind, extra):
    _oracle_kernels(monkeypatch)
    torch.manual_seed(0)
    ref, pat = _tiny(kind, **extra), _tiny(kind, **extra)
    ref.config._attn_implementation = pat.config._attn_implementation = "eager"
    pat.load_state_dict(ref.state_dict())
    bloth_b200.patch_model(pat, patch_norms=False, patch_attention=True, verbose=False)
    ids = torch.randint(0, 64, (2, 24), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        a, b = ref(ids).logits, pat(ids).logits
    assert float((a - b).abs().max()) < 1e-4


def test_fast_model_loads_a_local_checkpoint_and_patches_it(tmp_path):
    # FastModel.from_pretrained (reference patch.py:133-200) against a model and
    # tokenizer saved locally (no network); device_map=None keeps it on the CPU
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {"<unk>": 0, "<eos>": 1, **{f"w{i}": i + 2 for i in range(62)}}
    tk = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="<unk>",
                            eos_token="<eos>").save_pretrained(tmp_path)
    _tiny("qwen3").save_pretrained(tmp_path)
    model, tok = bloth_b200.FastModel.from_pretrained(str(tmp_path), device_map=None,
                                                      dtype=torch.float32)
    assert tok.pad_token == tok.eos_token == "<eos>"
    norms = [m for m in model.modules() if type(m).__name__ == "BlothRMSNorm"]
    assert len(norms) == 9  # 2 layers x (input, post-attention, q_norm, k_norm) + final
    assert next(model.parameters()).dtype == torch.float32
