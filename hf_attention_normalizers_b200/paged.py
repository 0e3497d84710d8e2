"""Paged-KV attention entry points (reference: hf_attention_normalizers/paged.py:1-318).

* ``paged_attention`` and ``paged_triton_attention`` keep the reference's
  signatures and validation messages and run the engine's paged kernels
  (``hfan::paged_fwd`` / ``hfan::paged_bwd``); cache-page gradients scatter
  back into the physical pages, accumulating where pages are shared.
* ``paged_cache_indices`` is the same host-side index helper.
* ``DifferentiablePagedCache`` / ``DifferentiablePagedCacheLayer`` are the
  HuggingFace cache with functional (out-of-place) page writes, so gradients
  reach the cache pages.
"""

from __future__ import annotations

from typing import Callable, Optional, Union

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _native as N
from . import ops


class DifferentiablePagedCacheLayer(CacheLayerMixin):
    """One layer of a paged cache whose writes keep the autograd graph."""

    def __init__(self, block_table: torch.Tensor, block_size: int, num_key_value_heads: int,
                 head_dim: int, dtype: torch.dtype, device: torch.device):
        super().__init__()
        if block_table.ndim != 2:
            raise ValueError("block_table must have shape [batch, max_blocks].")
        self.block_table = block_table.to(device=device, dtype=torch.long)
        self.block_size = block_size
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.device = device
        self.dtype = dtype
        self.max_batch_size = block_table.shape[0]
        self.max_cache_len = block_table.shape[1] * block_size
        self.cumulative_length = 0
        self.lazy_initialization(None)

    def lazy_initialization(self, key_states=None, value_states=None):
        pages = int(self.block_table.max().item()) + 1
        shape = (pages * self.block_size, self.num_key_value_heads, self.head_dim)
        self.keys = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.values = torch.zeros_like(self.keys)
        self.is_initialized = True

    def _physical(self, positions: torch.Tensor) -> torch.Tensor:
        pages = self.block_table[:, positions // self.block_size]
        return pages * self.block_size + positions.remainder(self.block_size)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor,
               cache_kwargs: Optional[dict] = None, *args, **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
        if key_states.shape != value_states.shape or key_states.ndim != 4:
            raise ValueError("K/V updates must have matching [batch, heads, sequence, dim] shapes.")
        if key_states.shape[:2] != (self.max_batch_size, self.num_key_value_heads):
            raise ValueError("K/V update batch or head count does not match the paged cache.")
        cache_kwargs = cache_kwargs or {}
        positions = cache_kwargs.get("cache_position")
        if positions is None:
            positions = torch.arange(self.cumulative_length, self.cumulative_length + key_states.shape[-2],
                                     device=self.device)
        positions = positions.to(device=self.device, dtype=torch.long)
        if positions.ndim != 1 or positions.numel() != key_states.shape[-2]:
            raise ValueError("cache_position must have one logical position per update token.")
        if int(positions.max().item()) >= self.max_cache_len:
            raise ValueError("cache_position exceeds the logical paged-cache capacity.")
        rows = self._physical(positions).reshape(-1)
        if torch.unique(rows).numel() != rows.numel():
            raise ValueError("Two batch entries cannot write the same physical cache page.")
        flat_k = key_states.transpose(1, 2).reshape(-1, self.num_key_value_heads, self.head_dim)
        flat_v = value_states.transpose(1, 2).reshape_as(flat_k)
        self.keys = torch.index_copy(self.keys, 0, rows, flat_k)
        self.values = torch.index_copy(self.values, 0, rows, flat_v)
        self.cumulative_length = max(self.cumulative_length, int(positions[-1].item()) + 1)
        read = self._physical(torch.arange(self.cumulative_length, device=self.device))
        return self.keys[read].permute(0, 2, 1, 3), self.values[read].permute(0, 2, 1, 3)

    def get_mask_sizes(self, cache_position) -> tuple[int, int]:
        if isinstance(cache_position, torch.Tensor):
            new_length = int(cache_position[-1].item()) + 1 if cache_position.numel() else self.cumulative_length
        else:
            new_length = self.cumulative_length + int(cache_position)
        return max(self.cumulative_length, new_length), 0

    def get_seq_length(self) -> int:
        return self.cumulative_length

    def get_max_cache_shape(self) -> int:
        return self.max_cache_len

    def reset(self) -> None:
        self.keys = torch.zeros_like(self.keys)
        self.values = torch.zeros_like(self.values)
        self.cumulative_length = 0


class DifferentiablePagedCache(Cache):
    """HuggingFace Cache of DifferentiablePagedCacheLayer, one per decoder layer."""

    def __init__(self, num_hidden_layers: int, block_table: torch.Tensor, block_size: int,
                 num_key_value_heads: int, head_dim: int, dtype: torch.dtype, device: torch.device):
        layers = [DifferentiablePagedCacheLayer(block_table, block_size, num_key_value_heads, head_dim,
                                                dtype, device) for _ in range(num_hidden_layers)]
        super().__init__(layers=layers)


def paged_cache_indices(block_table: torch.Tensor, sequence_lengths: torch.Tensor,
                        block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Physical token index and validity of every logical position, [batch, max_len]."""
    if block_table.ndim != 2:
        raise ValueError("block_table must have shape [batch, max_blocks].")
    if sequence_lengths.ndim != 1 or sequence_lengths.shape[0] != block_table.shape[0]:
        raise ValueError("sequence_lengths must have shape [batch].")
    if block_size <= 0:
        raise ValueError("block_size must be positive.")
    if bool((sequence_lengths <= 0).any()):
        raise ValueError("Every sequence length must be positive.")
    max_len = int(sequence_lengths.max().item())
    if max_len > block_table.shape[1] * block_size:
        raise ValueError("block_table does not contain enough blocks for sequence_lengths.")
    positions = torch.arange(max_len, device=block_table.device)
    physical = block_table[:, positions // block_size] * block_size + positions.remainder(block_size)
    valid = positions.unsqueeze(0) < sequence_lengths.unsqueeze(1)
    return physical, valid


def _normalizer_name(normalizer: Union[str, Callable[..., torch.Tensor]]) -> str:
    if isinstance(normalizer, str):
        if normalizer in N.NORMALIZER_IDS:
            return normalizer
        raise ValueError("paged attention supports 'softmax1', 'sparsemax', or 'entmax15'.")
    from . import vutils

    for name, fn in (("softmax1", vutils.softmax_1), ("sparsemax", vutils.sparsemax), ("entmax15", vutils.entmax15)):
        if normalizer is fn:
            return name
    raise ValueError("paged attention supports 'softmax1', 'sparsemax', or 'entmax15'.")


def _check_block_table(block_table, sequence_lengths, block_size, cache_tokens) -> int:
    """Eager-only bounds check of the block table; returns the max key length."""
    physical, _ = paged_cache_indices(block_table, sequence_lengths, block_size)
    if int(physical.max().item()) >= cache_tokens or int(physical.min().item()) < 0:
        raise ValueError("block_table references a block outside the physical cache.")
    return int(sequence_lengths.max().item())


def paged_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                    block_table: torch.Tensor, sequence_lengths: torch.Tensor, block_size: int,
                    normalizer: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                    scale: Optional[float] = None, is_causal: bool = True) -> torch.Tensor:
    """Differentiable paged attention over physical cache pages.

    query ``[batch, q_heads, q_len, dim]``; caches ``[num_blocks * block_size,
    kv_heads, dim]``; ``block_table`` ``[batch, max_blocks]``; causal masks are
    aligned to each sequence's end.  K/V gradients accumulate into their
    physical pages, including pages referenced more than once.
    """
    if query.ndim != 4:
        raise ValueError("query must have shape [batch, heads, sequence, dim].")
    if key_cache.ndim != 3 or value_cache.ndim != 3:
        raise ValueError("key_cache/value_cache must have shape [pages, heads, dim].")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache shapes must match.")
    if query.shape[0] != block_table.shape[0]:
        raise ValueError("query and block_table batch sizes must match.")
    if query.shape[-1] != key_cache.shape[-1]:
        raise ValueError("query and cache head dimensions must match.")
    if query.shape[1] % key_cache.shape[1] != 0:
        raise ValueError("query heads must be divisible by KV heads.")
    if not query.is_cuda or not key_cache.is_cuda or not value_cache.is_cuda:
        raise ValueError("paged_attention requires CUDA tensors.")
    name = _normalizer_name(normalizer)
    max_len = _check_block_table(block_table, sequence_lengths, block_size, key_cache.shape[0])
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    o, _ = ops.paged_fwd(query, key_cache, value_cache, block_table, sequence_lengths, int(block_size),
                         max_len, N.NORMALIZER_IDS[name], actual_scale, bool(is_causal))
    return o


def paged_triton_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                           block_table: torch.Tensor, sequence_lengths: torch.Tensor, block_size: int,
                           normalizer: str, scale: Optional[float] = None, is_causal: bool = True,
                           max_block_n: int = 4096, max_key_length: Optional[int] = None,
                           assume_unique_pages: bool = False) -> torch.Tensor:
    """Paged fused attention under the reference's name (paged.py:252-318).

    ``max_block_n`` and ``assume_unique_pages`` are accepted for
    compatibility: the engine's page gather and shared-page gradient
    accumulation need neither hint.
    """
    if normalizer not in {"softmax1", "softmax_1", "sparsemax", "entmax15"}:
        raise ValueError("paged_triton_attention supports 'softmax1', 'sparsemax', or 'entmax15'.")
    if not query.is_cuda or not key_cache.is_cuda or not value_cache.is_cuda:
        raise ValueError("paged_triton_attention requires CUDA tensors.")
    if query.ndim != 4:
        raise ValueError("query must have shape [batch, heads, sequence, dim].")
    if key_cache.ndim != 3 or key_cache.shape != value_cache.shape:
        raise ValueError("key_cache/value_cache must have matching [pages, heads, dim] shapes.")
    if query.shape[0] != block_table.shape[0]:
        raise ValueError("query and block_table batch sizes must match.")
    if query.shape[-1] != key_cache.shape[-1]:
        raise ValueError("query and cache head dimensions must match.")
    if query.shape[1] % key_cache.shape[1] != 0:
        raise ValueError("query heads must be divisible by KV heads.")
    if torch.compiler.is_compiling():
        if max_key_length is None:
            raise ValueError("Compiled paged attention requires static max_key_length.")
    else:
        max_len = _check_block_table(block_table, sequence_lengths, block_size, key_cache.shape[0])
        if max_key_length is None:
            max_key_length = max_len
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    o, _ = ops.paged_fwd(query, key_cache, value_cache, block_table, sequence_lengths, int(block_size),
                         int(max_key_length), N.NORMALIZER_IDS[normalizer], actual_scale, bool(is_causal))
    return o
