"""Row normalizers under the reference's ``vutils`` names
(reference: hf_attention_normalizers/vutils/{softmax1,entmax}.py).

On CUDA tensors these run the engine's row kernels (``hfan::rownorm_fwd``)
with closed-form backwards; CPU tensors raise ValueError (the engine has no
CPU path).  ``k`` (partial-sort size) is accepted for compatibility.
"""

from __future__ import annotations

import torch
from torch import nn

from ..ops import row_normalize


def softmax_1(input: torch.Tensor, dim: int = -1) -> torch.Tensor:
    r"""$\text(softmax)_1(x_i) = exp(x_i) / (1 + \sum_j exp(x_j))$"""
    return row_normalize(input, "softmax1", dim)


def sparsemax(X: torch.Tensor, dim: int = -1, k=None) -> torch.Tensor:
    """sparsemax: Euclidean projection of X onto the simplex along ``dim``."""
    return row_normalize(X, "sparsemax", dim)


def entmax15(X: torch.Tensor, dim: int = -1, k=None) -> torch.Tensor:
    """1.5-entmax along ``dim`` (as vutils: computed on (X - max) / 2)."""
    return row_normalize(X, "entmax15", dim)


softmax_1.__name__ = "softmax_1"


class Softmax_1(nn.Module):
    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, input):
        return softmax_1(input, self.dim)


class Sparsemax(nn.Module):
    def __init__(self, dim: int = -1, k=None):
        super().__init__()
        self.dim, self.k = dim, k

    def forward(self, X):
        return sparsemax(X, self.dim, self.k)


class Entmax15(nn.Module):
    def __init__(self, dim: int = -1, k=None):
        super().__init__()
        self.dim, self.k = dim, k

    def forward(self, X):
        return entmax15(X, self.dim, self.k)


__all__ = ["softmax_1", "sparsemax", "entmax15", "Softmax_1", "Sparsemax", "Entmax15"]
