"""``triton_sparsemax_attention`` / ``triton_entmax15_attention``
(reference: kernels/sparse_entmax_triton.py:180-199).

The reference's single-block kernel behind these names is superseded; the
names route to the same fused engine.  ``max_block_n`` is accepted for
compatibility (the engine has no key-length cap).
"""

from typing import Optional

import torch

from ._fused import fused_attention


def triton_sparsemax_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                               scale: Optional[float] = None, is_causal: bool = False,
                               max_block_n: int = 4096) -> torch.Tensor:
    return fused_attention(query, key, value, "sparsemax", scale, is_causal,
                           label="Triton sparse/entmax attention")


def triton_entmax15_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              scale: Optional[float] = None, is_causal: bool = False,
                              max_block_n: int = 4096) -> torch.Tensor:
    return fused_attention(query, key, value, "entmax15", scale, is_causal,
                           label="Triton sparse/entmax attention")
