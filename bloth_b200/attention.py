"""HuggingFace layer bindings: ``patch_model(..., patch_attention=True,
patch_residual=True)``.

The reference accepts ``patch_attention`` but does nothing with it
(bloth/bloth/patch.py:79-115; its model_patcher.py attention path cannot be
imported). Here every supported attention module gets a forward that routes
its q/k normalisation and rotary embedding through the sm_100a kernels:

* ``Qwen3Attention`` - ``q_norm`` / ``k_norm`` (RMSNorm over head_dim of the
  [B, S, H, D] projections) and ``apply_rotary_pos_emb`` become one
  ``fused_qk_norm_rope`` launch reading the layer's ``position_embeddings``
  tables (transformers models/qwen3/modeling_qwen3.py, Qwen3Attention.forward).
* ``LlamaAttention``, ``MistralAttention``, ``Qwen2Attention`` -
  ``apply_rotary_pos_emb`` of q and k becomes one ``apply_rope_qk`` launch.

The rest of the forward is HuggingFace's own code path, restated for the
transformers 5.x signature ``forward(hidden_states, position_embeddings,
attention_mask, past_key_values=None, **kwargs)``: the projections, the KV
cache update, the attention implementation the config selects (looked up in
the model's own modeling module), ``o_proj``. A module whose forward has
another signature, whose head_dim the kernels do not take (64, 128, 256) or
whose q and k norms differ in eps or weighting is left unpatched and reported.
The binding is per module instance; other models of the same class in the
process are untouched.

``patch_residual=True`` binds, per decoder layer (``LlamaDecoderLayer``,
``MistralDecoderLayer``, ``Qwen2DecoderLayer``, ``Qwen3DecoderLayer``), a
forward in which the attention block's residual add and the
``post_attention_layernorm`` that follows it are one ``fused_add_rms_norm``
launch (transformers models/llama/modeling_llama.py,
LlamaDecoderLayer.forward); the rest of the layer is HF's code.
"""
from __future__ import annotations

import inspect
import sys
import types
import warnings
from dataclasses import dataclass

import torch.nn as nn

from .kernels.add_rms_norm import fused_add_rms_norm
from .kernels.fused_norm_qkv_rope import fused_qk_norm_rope
from .kernels.rope import apply_rope_qk
from .modules import BlothRMSNorm
from .patch import _NORM_CLASS_NAMES, _NOT_RMS, _WEIGHT_OFFSETS, _module_eps

# class name -> (normalises q and k per head, source of the attention call's
# sliding_window argument: None (not passed), "module" or "config")
_ATTENTION_CLASSES = {
    "LlamaAttention": (False, None),
    "MistralAttention": (False, "config"),
    "Qwen2Attention": (False, "module"),
    "Qwen3Attention": (True, "module"),
}
_FORWARD_PARAMS = ["self", "hidden_states", "position_embeddings", "attention_mask",
                   "past_key_values", "kwargs"]
_HEAD_DIMS = (64, 128, 256)


@dataclass(frozen=True)
class _Binding:
    norms: bool
    window: str | None


def _norm_params(norm: nn.Module):
    """(weight, eps, weight_offset) of an RMSNorm the kernels can apply, or
    None: a BlothRMSNorm, or an HF norm on the recognised list."""
    if isinstance(norm, BlothRMSNorm):
        return norm.weight, float(norm.eps), norm.weight_offset
    cls = type(norm).__name__
    w = getattr(norm, "weight", None)
    if cls in _NORM_CLASS_NAMES and cls not in _NOT_RMS and isinstance(w, nn.Parameter) \
            and w.dim() == 1:
        return w, float(_module_eps(norm)), _WEIGHT_OFFSETS.get(cls, 0.0)
    return None


def _attention_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                       past_key_values=None, **kwargs):
    """HF 5.x attention forward with the q/k norm + RoPE step on the kernels."""
    bind = self._bloth_attention
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, self.head_dim)
    q = self.q_proj(hidden_states).view(hidden_shape)
    k = self.k_proj(hidden_states).view(hidden_shape)
    v = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    cos, sin = position_embeddings
    if bind.norms:
        wq, eps, off = _norm_params(self.q_norm)
        wk = _norm_params(self.k_norm)[0]
        q, k = fused_qk_norm_rope(q, k, wq, wk, eps=eps, cos=cos, sin=sin, weight_offset=off)
    else:
        q, k = apply_rope_qk(q, k, cos=cos, sin=sin)
    q, k = q.transpose(1, 2), k.transpose(1, 2)
    if past_key_values is not None:
        k, v = past_key_values.update(k, v, self.layer_idx)
    hf = sys.modules[type(self).__module__]
    attention_interface = hf.ALL_ATTENTION_FUNCTIONS.get_interface(
        self.config._attn_implementation, hf.eager_attention_forward)
    extra = {}
    if bind.window == "module":
        extra["sliding_window"] = self.sliding_window
    elif bind.window == "config":
        extra["sliding_window"] = getattr(self.config, "sliding_window", None)
    attn_output, attn_weights = attention_interface(
        self, q, k, v, attention_mask,
        dropout=0.0 if not self.training else self.attention_dropout,
        scaling=self.scaling, **extra, **kwargs)
    attn_output = attn_output.reshape(*input_shape, -1).contiguous()
    attn_output = self.o_proj(attn_output)
    return attn_output, attn_weights


def _why_not(module: nn.Module, norms: bool) -> str | None:
    """Reason the module cannot take the binding, or None."""
    params = list(inspect.signature(type(module).forward).parameters)
    if params != _FORWARD_PARAMS:
        return f"forward{tuple(params[1:])} is not the transformers 5.x signature"
    hf = sys.modules.get(type(module).__module__)
    if hf is None or not hasattr(hf, "ALL_ATTENTION_FUNCTIONS") or \
            not hasattr(hf, "eager_attention_forward"):
        return "its modeling module has no attention-function registry"
    if getattr(module, "head_dim", None) not in _HEAD_DIMS:
        return f"head_dim {getattr(module, 'head_dim', None)} is not one of {_HEAD_DIMS}"
    if norms:
        pq = _norm_params(getattr(module, "q_norm", None))
        pk = _norm_params(getattr(module, "k_norm", None))
        if pq is None or pk is None:
            return "q_norm / k_norm are not recognised RMSNorms"
        if pq[1:] != pk[1:]:
            return "q_norm and k_norm differ in eps or weighting"
        if pq[0].shape[0] != module.head_dim or pk[0].shape[0] != module.head_dim:
            return "q_norm / k_norm do not normalise over head_dim"
    return None


def patch_attention_layers(model: nn.Module, verbose: bool = True) -> int:
    """Binds the fused forward to every supported attention module of model;
    returns how many were bound."""
    bound, skipped = 0, []
    for name, module in model.named_modules():
        spec = _ATTENTION_CLASSES.get(type(module).__name__)
        if spec is None or hasattr(module, "_bloth_attention"):
            continue
        reason = _why_not(module, spec[0])
        if reason is not None:
            skipped.append(f"{name}: {reason}")
            continue
        module._bloth_attention = _Binding(norms=spec[0], window=spec[1])
        module.forward = types.MethodType(_attention_forward, module)
        bound += 1
    if skipped:
        warnings.warn("[Bloth] attention left unpatched - " + "; ".join(skipped[:4]) +
                      (f" (+{len(skipped) - 4} more)" if len(skipped) > 4 else ""))
    if verbose and bound > 0:
        print(f"[Bloth] Patched {bound} attention layer(s) -> fused q/k norm + RoPE")
    return bound


# ------------------------------------------------- decoder layer: residual add
_DECODER_CLASSES = {"LlamaDecoderLayer", "MistralDecoderLayer", "Qwen2DecoderLayer",
                    "Qwen3DecoderLayer"}
_DECODER_PARAMS = ["self", "hidden_states", "attention_mask", "position_ids", "past_key_values",
                   "use_cache", "position_embeddings", "kwargs"]


def _decoder_layer_forward(self, hidden_states, attention_mask=None, position_ids=None,
                           past_key_values=None, use_cache=False, position_embeddings=None,
                           **kwargs):
    """HF 5.x decoder layer with residual add + post-attention norm fused."""
    residual = hidden_states
    hidden_states = self.input_layernorm(hidden_states)
    hidden_states, _ = self.self_attn(
        hidden_states=hidden_states, attention_mask=attention_mask, position_ids=position_ids,
        past_key_values=past_key_values, use_cache=use_cache,
        position_embeddings=position_embeddings, **kwargs)
    w, eps, off = _norm_params(self.post_attention_layernorm)
    hidden_states, residual = fused_add_rms_norm(hidden_states, residual, w, eps, off)
    hidden_states = self.mlp(hidden_states)
    return residual + hidden_states


def patch_decoder_layers(model: nn.Module, verbose: bool = True) -> int:
    """Binds the fused residual forward to every supported decoder layer;
    returns how many were bound."""
    bound, skipped = 0, []
    for name, module in model.named_modules():
        if type(module).__name__ not in _DECODER_CLASSES or "forward" in module.__dict__:
            continue
        params = list(inspect.signature(type(module).forward).parameters)
        if params != _DECODER_PARAMS:
            skipped.append(f"{name}: forward{tuple(params[1:])} is not the transformers 5.x "
                           "signature")
            continue
        if _norm_params(getattr(module, "post_attention_layernorm", None)) is None:
            skipped.append(f"{name}: post_attention_layernorm is not a recognised RMSNorm")
            continue
        module.forward = types.MethodType(_decoder_layer_forward, module)
        bound += 1
    if skipped:
        warnings.warn("[Bloth] decoder layers left unpatched - " + "; ".join(skipped[:4]) +
                      (f" (+{len(skipped) - 4} more)" if len(skipped) > 4 else ""))
    if verbose and bound > 0:
        print(f"[Bloth] Patched {bound} decoder layer(s) -> fused residual add + RMSNorm")
    return bound
