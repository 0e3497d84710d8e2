"""``paged_hopper_sparse_attention`` (reference: kernels/paged_sparse_entmax_hopper.py:464-496)."""

from typing import Optional

import torch

from .. import _native as N
from .paged_softmax1_hopper import _paged


def paged_hopper_sparse_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                                  block_table: torch.Tensor, sequence_lengths: torch.Tensor, page_size: int,
                                  normalizer: str, scale: Optional[float] = None, is_causal: bool = True,
                                  block_n: int = 128, bisection_steps: int = 24,
                                  max_key_length: Optional[int] = None,
                                  assume_unique_pages: bool = False) -> torch.Tensor:
    if normalizer not in {"sparsemax", "entmax15"}:
        raise ValueError("normalizer must be 'sparsemax' or 'entmax15'.")
    if not query.is_cuda or not key_cache.is_cuda or not value_cache.is_cuda:
        raise ValueError("Paged Hopper attention requires CUDA tensors.")
    if key_cache.shape != value_cache.shape or key_cache.ndim != 3:
        raise ValueError("K/V caches must have matching [physical_tokens, kv_heads, dim] shapes.")
    if query.shape[0] != block_table.shape[0] or query.shape[0] != sequence_lengths.shape[0]:
        raise ValueError("Batch dimensions must match.")
    if query.shape[1] % key_cache.shape[1] != 0:
        raise ValueError("Query heads must be divisible by KV heads.")
    return _paged(query, key_cache, value_cache, block_table, sequence_lengths, page_size,
                  N.NORMALIZER_IDS[normalizer], scale, is_causal, max_key_length)
