"""B200-native fused normalizer attention (softmax1 / sparsemax / entmax15).

Drop-in for the public API of ``hf_attention_normalizers``
(reference: hf_attention_normalizers/__init__.py:1-57): the same 25 names,
backed by hand-written sm_100a CUDA kernels in ``_lib/libhfan.so``.
"""

from .backends import (
    AttentionReplacementPolicy,
    Qwen3AttentionExtra,
    Qwen3AttentionExtrea,
    apply_softmax1_attention,
    apply_softmax_attention,
    from_pretrained_with_registered_softmax_attention,
    from_pretrained_with_softmax_attention,
    register_attention_replacement_policy,
    register_entmax15_attention_backends,
    register_softmax1_attention_backends,
    register_softmax_attention_backends,
    register_sparsemax_attention_backends,
    replace_attention_modules,
    replace_qwen3_attention_modules,
    set_softmax_attention_backend,
    softmax_attention_backend_name,
    supported_attention_policies,
    triton_entmax15_attention_forward,
    triton_sparsemax_attention_forward,
)
from .paged import (
    DifferentiablePagedCache,
    DifferentiablePagedCacheLayer,
    paged_attention,
    paged_cache_indices,
    paged_triton_attention,
)
from .varlen import varlen_hopper_attention

__all__ = [
    "AttentionReplacementPolicy",
    "Qwen3AttentionExtra",
    "Qwen3AttentionExtrea",
    "apply_softmax1_attention",
    "apply_softmax_attention",
    "from_pretrained_with_registered_softmax_attention",
    "from_pretrained_with_softmax_attention",
    "register_attention_replacement_policy",
    "register_entmax15_attention_backends",
    "register_softmax1_attention_backends",
    "register_softmax_attention_backends",
    "register_sparsemax_attention_backends",
    "replace_attention_modules",
    "replace_qwen3_attention_modules",
    "set_softmax_attention_backend",
    "softmax_attention_backend_name",
    "supported_attention_policies",
    "triton_entmax15_attention_forward",
    "triton_sparsemax_attention_forward",
    "paged_attention",
    "paged_cache_indices",
    "paged_triton_attention",
    "DifferentiablePagedCache",
    "DifferentiablePagedCacheLayer",
    "varlen_hopper_attention",
]
