"""``hopper_softmax1_attention`` (reference: kernels/softmax1_hopper.py:412-452)."""

from typing import Optional

import torch

from ._fused import fused_attention


def hopper_softmax1_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              scale: Optional[float] = None, is_causal: bool = False,
                              window_left: Optional[int] = None, block_n: int = 128,
                              dropout_p: float = 0.0) -> torch.Tensor:
    """Fused softmax1 attention, [B,H,S,D] in and out.  ``block_n`` is accepted
    for signature compatibility; tile shapes are fixed by the kernel."""
    return fused_attention(query, key, value, "softmax1", scale, is_causal, window_left, dropout_p,
                           label="Softmax1 Hopper attention")
