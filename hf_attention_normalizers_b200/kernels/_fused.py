"""Shared entry for the dense fused kernels behind the reference's kernel names.

Mirrors the argument checks of ``kernels/softmax1_hopper.py:412-452`` and
``kernels/sparse_entmax_hopper.py:428-501`` (same messages), then calls the
``hfan::attn_fwd`` op.  GQA is handled inside the kernel: ``key``/``value``
may have fewer heads than ``query`` (the reference required equal heads and
expanded GQA with ``repeat_kv`` before the call).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _native as N
from .. import ops


def check_dense(query, key, value, label: str) -> None:
    if not query.is_cuda or not key.is_cuda or not value.is_cuda:
        raise ValueError(f"{label} requires CUDA tensors.")
    if (query.ndim != 4 or key.ndim != 4 or key.shape != value.shape
            or query.shape[0] != key.shape[0] or query.shape[1] % key.shape[1] != 0):
        raise ValueError("Expected compatible Q/K/V tensors shaped [batch, heads, sequence, dim].")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError("Q/K/V head dimensions must match.")
    if query.shape[-1] > 256:
        raise ValueError("head_dim larger than 256 is not supported.")


def check_dropout(dropout_p: float, query: Optional[torch.Tensor] = None) -> None:
    if not 0.0 <= dropout_p < 1.0:
        raise ValueError("dropout_p must be in [0, 1).")
    if dropout_p > 0.0 and query is not None and (
            query.dtype not in (torch.bfloat16, torch.float16) or query.shape[-1] not in (64, 128)):
        raise NotImplementedError("Fused attention dropout needs float16/bfloat16 inputs with head_dim 64 or 128.")


def dropout_seed(query: torch.Tensor, dropout_p: float) -> Optional[torch.Tensor]:
    """One value from PyTorch's CUDA RNG, kept on the device for the forward and
    the backward (kernels/softmax1_hopper.py:434-441): re-seeding PyTorch
    reproduces the same dropout mask."""
    if dropout_p == 0.0:
        return None
    return torch.empty((), device=query.device, dtype=torch.int64).random_(2 ** 31 - 1)


def fused_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, normalizer: str,
                    scale: Optional[float] = None, is_causal: bool = False,
                    window_left: Optional[int] = None, dropout_p: float = 0.0,
                    label: str = "Hopper attention", out_bshd: bool = False) -> torch.Tensor:
    """Dense fused attention; returns [B, Hq, S, D] (or [B, S, Hq, D] if ``out_bshd``)."""
    check_dense(query, key, value, label)
    check_dropout(dropout_p, query)
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    window = -1 if window_left is None else int(window_left)
    o = ops.attn_fwd(query, key, value, N.NORMALIZER_IDS[normalizer], actual_scale, bool(is_causal),
                           window, bool(out_bshd), float(dropout_p), dropout_seed(query, dropout_p))[0]
    return o
