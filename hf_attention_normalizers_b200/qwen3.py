"""Qwen3 attention module with a pluggable normalizer and the model-surgery
helpers (reference: hf_attention_normalizers/backends.py:1171-1478).

This is model plumbing around the fused engine: projections, QK-RMSNorm and
RoPE come from transformers; the attention call goes through the registered
AttentionInterface name.
"""

from __future__ import annotations

from typing import Callable, Optional, Union

import torch
from torch import nn
from transformers.models.qwen3.modeling_qwen3 import Qwen3Config, Qwen3RMSNorm, apply_rotary_pos_emb

from . import backends as B


class Qwen3AttentionExtrea(nn.Module):
    """Qwen3 attention with pluggable attention backend and pluggable softmax."""

    def __init__(self, config: Qwen3Config, layer_idx: int,
                 softmax_fn: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                 attn_implementation: Optional[str] = None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.num_key_value_groups = config.num_attention_heads // config.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        self.attention_dropout = config.attention_dropout
        self.is_causal = True
        self.softmax_fn = B.resolve_softmax_fn(softmax_fn)
        self.softmax_name = softmax_fn if isinstance(softmax_fn, str) else getattr(softmax_fn, "__name__", "callable")
        self.attn_implementation = attn_implementation
        bias = config.attention_bias
        self.q_proj = nn.Linear(config.hidden_size, config.num_attention_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, config.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, config.num_key_value_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(config.num_attention_heads * self.head_dim, config.hidden_size, bias=bias)
        self.q_norm = Qwen3RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = Qwen3RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        layer_types = getattr(config, "layer_types", None)
        sliding = layer_types is not None and layer_types[layer_idx] == "sliding_attention"
        self.sliding_window = config.sliding_window if sliding else None

    def forward(self, hidden_states: torch.Tensor, position_embeddings: tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor], past_key_values=None, cache_position=None, **kwargs):
        if past_key_values is None:
            past_key_values = kwargs.pop("past_key_value", None)
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        self.to(device=hidden_states.device, dtype=hidden_states.dtype)
        query_states = self.q_norm(self.q_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
        key_states = self.k_norm(self.k_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
        value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        cos, sin = position_embeddings
        query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)
        if past_key_values is not None:
            cache_kwargs = {"sin": sin, "cos": cos, "cache_position": cache_position}
            key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx, cache_kwargs)
        attn_implementation = (kwargs.pop("attn_implementation", None) or self.attn_implementation
                               or getattr(self.config, "_attn_implementation", "eager"))
        if B._uses_custom_softmax(self.softmax_name) and not B._is_allowed_custom_softmax_backend(
                self.softmax_name, attn_implementation):
            valid = ", ".join(sorted(B.CUSTOM_ATTENTION_FUNCTIONS))
            raise ValueError(f"{self.softmax_name} requires a custom-softmax attention backend. "
                             f"Use one of: {valid}. Got: {attn_implementation}")
        attention_interface = B.get_attention_forward(attn_implementation)
        attn_output, attn_weights = attention_interface(
            self, query_states, key_states, value_states, attention_mask, softmax_fn=self.softmax_fn,
            dropout=0.0 if not self.training else self.attention_dropout, scaling=self.scaling,
            sliding_window=self.sliding_window, **kwargs)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return self.o_proj(attn_output), attn_weights


Qwen3AttentionExtra = Qwen3AttentionExtrea


def _matches_qwen3_attention(module: nn.Module) -> bool:
    is_qwen3 = module.__class__.__name__ in {"Qwen3Attention", "Qwen3AttentionExtrea", "Qwen3AttentionExtra"}
    has_proj = all(hasattr(module, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj"))
    return is_qwen3 and has_proj and hasattr(module, "config") and hasattr(module, "layer_idx")


def _build_qwen3_attention_replacement(module: nn.Module, softmax_fn="softmax1", attn_implementation: str = "sdpa"):
    replacement = Qwen3AttentionExtrea(module.config, module.layer_idx, softmax_fn=softmax_fn,
                                       attn_implementation=attn_implementation)
    replacement.load_state_dict(module.state_dict(), strict=False)
    first = next(module.parameters())
    replacement.to(device=first.device, dtype=first.dtype)
    replacement.train(module.training)
    return replacement


ATTENTION_REPLACEMENT_POLICIES: dict[str, B.AttentionReplacementPolicy] = {
    "qwen3": B.AttentionReplacementPolicy(name="qwen3", matches=_matches_qwen3_attention,
                                          build=_build_qwen3_attention_replacement),
}


def register_attention_replacement_policy(policy: B.AttentionReplacementPolicy) -> None:
    ATTENTION_REPLACEMENT_POLICIES[policy.name] = policy


def supported_attention_policies() -> tuple[str, ...]:
    return tuple(sorted(ATTENTION_REPLACEMENT_POLICIES))


def replace_attention_modules(model: nn.Module, softmax_fn="softmax1", attn_implementation: str = "sdpa",
                              policy_names: Optional[tuple[str, ...]] = None) -> int:
    """Replace supported attention modules in place; returns how many were replaced."""
    policies = ATTENTION_REPLACEMENT_POLICIES
    if policy_names is not None:
        policies = {n: ATTENTION_REPLACEMENT_POLICIES[n] for n in policy_names}
    replaced = 0
    for name, child in list(model.named_children()):
        replacement = None
        for policy in policies.values():
            if policy.matches(child):
                replacement = policy.build(child, softmax_fn, attn_implementation)
                break
        if replacement is not None:
            setattr(model, name, replacement)
            replaced += 1
        else:
            replaced += replace_attention_modules(child, softmax_fn, attn_implementation, policy_names)
    return replaced


def replace_qwen3_attention_modules(model: nn.Module, softmax_fn="softmax1", attn_implementation: str = "sdpa") -> int:
    return replace_attention_modules(model, softmax_fn=softmax_fn, attn_implementation=attn_implementation,
                                     policy_names=("qwen3",))


def apply_softmax_attention(model: nn.Module, softmax_fn="softmax1", attn_implementation: str = "sdpa") -> nn.Module:
    replaced = replace_attention_modules(model, softmax_fn=softmax_fn, attn_implementation=attn_implementation)
    if replaced == 0:
        supported = ", ".join(sorted(ATTENTION_REPLACEMENT_POLICIES))
        raise ValueError(f"No supported attention modules found. Registered policies: {supported}")
    if hasattr(model, "config"):
        model.config._attn_implementation = attn_implementation
    return model


def apply_softmax1_attention(model: nn.Module, attn_implementation: str = "sdpa") -> nn.Module:
    return apply_softmax_attention(model, softmax_fn="softmax1", attn_implementation=attn_implementation)


def from_pretrained_with_softmax_attention(model_name_or_path: str, softmax_fn="softmax1",
                                           attn_implementation: str = "sdpa", auto_model_cls=None,
                                           **from_pretrained_kwargs) -> nn.Module:
    if auto_model_cls is None:
        from transformers import AutoModelForCausalLM as auto_model_cls
    model = auto_model_cls.from_pretrained(model_name_or_path, **from_pretrained_kwargs)
    return apply_softmax_attention(model, softmax_fn=softmax_fn, attn_implementation=attn_implementation)


def from_pretrained_with_registered_softmax_attention(model_name_or_path: str, softmax_fn="softmax1",
                                                      base_backend: str = "sdpa", mode: str = "strict",
                                                      fallback_backend: str = "sdpa", auto_model_cls=None,
                                                      **from_pretrained_kwargs) -> nn.Module:
    B._register_for(softmax_fn, mode, fallback_backend)
    from_pretrained_kwargs.setdefault("attn_implementation",
                                      B.softmax_attention_backend_name(base_backend, softmax_fn))
    if auto_model_cls is None:
        from transformers import AutoModelForCausalLM as auto_model_cls
    return auto_model_cls.from_pretrained(model_name_or_path, **from_pretrained_kwargs)
