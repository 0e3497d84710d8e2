"""``varlen_hopper_sparse_attention`` (reference: kernels/varlen_sparse_entmax_hopper.py:141-147)."""

from typing import Optional

import torch

from .. import _native as N
from .. import ops


def varlen_hopper_sparse_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                   cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, normalizer: str,
                                   max_seqlen_q: int, max_seqlen_k: int, scale: Optional[float] = None,
                                   is_causal: bool = True, block_n: int = 128,
                                   bisection_steps: int = 24) -> torch.Tensor:
    if query.shape[-1] > 256:
        raise ValueError("head_dim larger than 256 is not supported.")
    if normalizer not in {"sparsemax", "entmax15"}:
        raise ValueError("normalizer must be sparsemax or entmax15.")
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    o = ops.varlen_fwd(query, key, value, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q),
                       int(max_seqlen_k), N.NORMALIZER_IDS[normalizer], actual_scale, bool(is_causal))[0]
    return o
