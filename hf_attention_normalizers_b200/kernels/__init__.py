"""Kernel-level entry points under the reference's names
(reference: hf_attention_normalizers/kernels/__init__.py:1-18)."""

from .paged_softmax1_hopper import paged_hopper_softmax1_attention
from .paged_sparse_entmax_hopper import paged_hopper_sparse_attention
from .softmax1_hopper import hopper_softmax1_attention
from .sparse_entmax_hopper import hopper_entmax15_attention, hopper_sparsemax_attention
from .sparse_entmax_triton import triton_entmax15_attention, triton_sparsemax_attention

__all__ = [
    "hopper_entmax15_attention",
    "hopper_softmax1_attention",
    "hopper_sparsemax_attention",
    "paged_hopper_softmax1_attention",
    "paged_hopper_sparse_attention",
    "triton_entmax15_attention",
    "triton_sparsemax_attention",
]
