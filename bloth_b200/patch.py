"""HuggingFace model patcher: swaps every recognised RMSNorm for BlothRMSNorm.

Same entry points and behaviour as the reference's bloth/bloth/patch.py:
``patch_model(model, patch_norms=True, patch_attention=False, verbose=True)``
(:79-115) walks the module tree and replaces every module whose class name is
in ``_NORM_CLASS_NAMES`` (:26-43) by a ``BlothRMSNorm`` that shares the
original ``weight`` Parameter (:46-76), so state_dict keys are unchanged;
``FastModel.from_pretrained`` (:133-200) loads a model and patches it.

Two corrections to the reference's norm swap, both silent output changes
there: Gemma-family norms compute x_hat * (1 + w) (transformers
GemmaRMSNorm.forward), so they become ``BlothRMSNorm(weight_offset=1.0)``
rather than an x_hat * w norm; and ``CohereLayerNorm``, although on the
reference's list, subtracts the mean (it is a LayerNorm), so it is left in
place. ``patch_attention=True`` (a no-op in the reference) routes supported
attention modules through the fused kernels (``bloth_b200.attention``).
"""
from __future__ import annotations

import warnings

import torch
import torch.nn as nn

from .modules import BlothRMSNorm

# Every RMSNorm class name across the supported HF models (reference patch.py:26-43).
_NORM_CLASS_NAMES = {
    "LlamaRMSNorm",
    "MistralRMSNorm",
    "MixtralRMSNorm",
    "QwenRMSNorm",
    "Qwen2RMSNorm",
    "Qwen3RMSNorm",
    "GemmaRMSNorm",
    "Gemma2RMSNorm",
    "PhiRMSNorm",
    "Phi3RMSNorm",
    "FalconRMSNorm",
    "MptRMSNorm",
    "T5LayerNorm",
    "CohereLayerNorm",
    "OlmoRMSNorm",
    "DeepseekRMSNorm",
}

# Norms on the list above whose weight enters as (1 + w).
_WEIGHT_OFFSETS = {"GemmaRMSNorm": 1.0, "Gemma2RMSNorm": 1.0}

# Names on the reference's list that are not RMSNorms and are left in place.
_NOT_RMS = {"CohereLayerNorm"}


def _module_eps(module: nn.Module) -> float:
    """eps lookup order of the reference (patch.py:61-63)."""
    return getattr(module, "eps", getattr(module, "variance_epsilon",
                                          getattr(module, "norm_eps", 1e-6)))


def _replace_norm_layers(model: nn.Module, verbose: bool = True) -> int:
    """Replaces every recognised norm with a BlothRMSNorm sharing its weight."""
    replaced = 0
    mod_dict = dict(model.named_modules())
    for name, module in list(mod_dict.items()):
        cls = type(module).__name__
        if cls not in _NORM_CLASS_NAMES or cls in _NOT_RMS:
            continue
        weight = getattr(module, "weight", None)
        if not isinstance(weight, nn.Parameter) or weight.dim() != 1:
            continue
        parts = name.rsplit(".", 1)
        parent = mod_dict[parts[0]] if len(parts) == 2 else model
        attr = parts[-1]
        hidden_size = module.weight.shape[0]
        norm = BlothRMSNorm(hidden_size, _module_eps(module),
                            weight_offset=_WEIGHT_OFFSETS.get(cls, 0.0)).to(
            device=module.weight.device, dtype=module.weight.dtype)
        norm.weight = module.weight  # share the Parameter, no copy
        setattr(parent, attr, norm)
        replaced += 1
    if verbose and replaced > 0:
        print(f"[Bloth] Replaced {replaced} norm layer(s) -> BlothRMSNorm")
    return replaced


def patch_model(model: nn.Module, patch_norms: bool = True, patch_attention: bool = False,
                verbose: bool = True, patch_residual: bool = False) -> nn.Module:
    """Applies the Bloth kernels to a HuggingFace model in place and returns it.

    patch_norms: replace RMSNorm layers (reference behaviour).
    patch_attention: route the q/k normalisation and rotary embedding of
        supported attention modules through the fused kernels (Qwen3: one
        fused_qk_norm_rope launch; Llama / Mistral / Qwen2: one RoPE launch
        for q and k). The reference accepts this flag and does nothing.
    patch_residual: fuse each decoder layer's attention residual add with its
        post_attention_layernorm (fused_add_rms_norm). Not in the reference.
    """
    if verbose:
        print(f"\n[Bloth] Patching: {type(model).__name__}")
        if torch.cuda.is_available():
            p = torch.cuda.get_device_properties(torch.cuda.current_device())
            print(f"[Bloth] GPU: {p.name} | sm_{p.major}{p.minor}")
    total = 0
    if patch_norms:
        total += _replace_norm_layers(model, verbose)
    if patch_attention:
        from .attention import patch_attention_layers
        total += patch_attention_layers(model, verbose)
    if patch_residual:
        from .attention import patch_decoder_layers
        total += patch_decoder_layers(model, verbose)
    if total == 0 and verbose:
        warnings.warn("[Bloth] No layers patched. Architecture may not be recognised. "
                      "You can still use bloth_b200.kernels.* directly.")
    elif verbose:
        print(f"[Bloth] Total: {total} patch(es).\n")
    return model


class FastModel:
    """Loads a HuggingFace causal LM and patches it (reference: patch.py:118-200)."""

    @staticmethod
    def from_pretrained(model_name: str, max_seq_length: int = 4096, dtype=None,
                        load_in_4bit: bool = False, load_in_8bit: bool = False,
                        device_map: str = "auto", trust_remote_code: bool = False,
                        patch_attention: bool = False, **kwargs):
        try:
            from transformers import AutoModelForCausalLM, AutoTokenizer
        except ImportError:
            raise ImportError("pip install transformers") from None
        if dtype is None:
            if torch.cuda.is_available():
                major = torch.cuda.get_device_properties(torch.cuda.current_device()).major
                dtype = torch.bfloat16 if major >= 8 else torch.float16
            else:
                dtype = torch.float32
        quant_cfg = None
        if load_in_4bit or load_in_8bit:
            try:
                from transformers import BitsAndBytesConfig
                quant_cfg = BitsAndBytesConfig(load_in_4bit=load_in_4bit,
                                               load_in_8bit=load_in_8bit,
                                               bnb_4bit_compute_dtype=dtype,
                                               bnb_4bit_use_double_quant=True,
                                               bnb_4bit_quant_type="nf4")
            except ImportError:
                warnings.warn("[Bloth] bitsandbytes not installed - quantization skipped.")
        print(f"[Bloth] Loading {model_name} ...")
        model = AutoModelForCausalLM.from_pretrained(model_name, torch_dtype=dtype,
                                                     device_map=device_map,
                                                     quantization_config=quant_cfg,
                                                     trust_remote_code=trust_remote_code,
                                                     **kwargs)
        tokenizer = AutoTokenizer.from_pretrained(model_name, trust_remote_code=trust_remote_code)
        if tokenizer.pad_token is None:
            tokenizer.pad_token = tokenizer.eos_token
        model = patch_model(model, patch_attention=patch_attention, verbose=True)
        return model, tokenizer
