"""``paged_hopper_softmax1_attention`` (reference: kernels/paged_softmax1_hopper.py:352-375)."""

from typing import Optional

import torch

from .. import _native as N
from .. import ops


def paged_hopper_softmax1_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                                    block_table: torch.Tensor, sequence_lengths: torch.Tensor, page_size: int,
                                    scale: Optional[float] = None, is_causal: bool = True, block_n: int = 128,
                                    max_key_length: Optional[int] = None,
                                    assume_unique_pages: bool = False) -> torch.Tensor:
    if not query.is_cuda or not key_cache.is_cuda or not value_cache.is_cuda:
        raise ValueError("Paged Softmax1 attention requires CUDA tensors.")
    if key_cache.shape != value_cache.shape or query.shape[1] % key_cache.shape[1] != 0:
        raise ValueError("Incompatible Q/K/V head shapes.")
    return _paged(query, key_cache, value_cache, block_table, sequence_lengths, page_size, N.SOFTMAX1,
                  scale, is_causal, max_key_length)


def _paged(query, key_cache, value_cache, block_table, sequence_lengths, page_size, normalizer, scale,
           is_causal, max_key_length):
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    if max_key_length is None:
        max_key_length = int(sequence_lengths.max().item())
    o, _ = ops.paged_fwd(query, key_cache, value_cache, block_table, sequence_lengths, int(page_size),
                         int(max_key_length), normalizer, actual_scale, bool(is_causal))
    return o
