"""``hopper_sparsemax_attention`` / ``hopper_entmax15_attention``
(reference: kernels/sparse_entmax_hopper.py:472-501).

``bisection_steps`` and ``block_n`` are accepted for signature compatibility;
the engine solves the threshold exactly (no bisection).
"""

from typing import Optional

import torch

from ._fused import fused_attention


def hopper_sparsemax_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                               scale: Optional[float] = None, is_causal: bool = False,
                               window_left: Optional[int] = None, block_n: int = 128,
                               bisection_steps: int = 24, dropout_p: float = 0.0) -> torch.Tensor:
    return fused_attention(query, key, value, "sparsemax", scale, is_causal, window_left, dropout_p,
                           label="Hopper sparse attention")


def hopper_entmax15_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              scale: Optional[float] = None, is_causal: bool = False,
                              window_left: Optional[int] = None, block_n: int = 128,
                              bisection_steps: int = 24, dropout_p: float = 0.0) -> torch.Tensor:
    return fused_attention(query, key, value, "entmax15", scale, is_causal, window_left, dropout_p,
                           label="Hopper sparse attention")
