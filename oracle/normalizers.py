"""Row normalizers (softmax1, sparsemax, 1.5-entmax) in numpy.  TEST INFRASTRUCTURE.

Each function restates the reference's eager implementation step by step so
that its rounding behaviour is the same family (sort + cumsum, max shift):

* softmax1   -- ``hf_attention_normalizers/vutils/softmax1.py:4-28``
  (``softmax_n_shifted_zeros`` with n=1): shift by the row max m, numerator
  exp(x-m), denominator sum(exp(x-m)) + exp(-m).
* sparsemax  -- ``vutils/entmax.py:35-79`` (``_sparsemax_threshold_and_support``)
  and ``:136-157`` (``SparsemaxFunction``): max shift, full descending sort,
  cumsum-1, support = rho*z_sorted > cumsum-1, tau = (cumsum-1)[k-1]/k,
  p = max(z - tau, 0).  Backward: dX = 1[p>0] (dY - sum_{p>0} dY / k).
* entmax15   -- ``vutils/entmax.py:82-133`` and ``:160-183``
  (``Entmax15Function``): z = (x - max)/2, sorted running mean / mean of
  squares, tau_rho = mean - sqrt(max((1 - ss)/rho, 0)), support =
  #{tau_rho <= z_sorted}, p = max(z - tau*, 0)^2.  Backward with g = sqrt(p):
  dX = g dY - (sum g dY / sum g) g.  Note: exactly like the reference, the
  backward does not apply the 1/2 factor of the z = x/2 rescaling.

All functions operate on the last axis.  They are written for clarity, not
speed; masked entries are expected to hold ``finfo(dtype).min`` exactly as the
reference's eager attention fills them (``backends.py:64-68``).
"""

from __future__ import annotations

import numpy as np


def _rho(n: int, dtype) -> np.ndarray:
    return np.arange(1, n + 1, dtype=dtype)


def softmax1(x: np.ndarray) -> np.ndarray:
    """softmax_1 along the last axis (reference vutils/softmax1.py:4-28)."""
    m = x.max(axis=-1, keepdims=True)
    with np.errstate(over="ignore", under="ignore"):
        num = np.exp(x - m)
        den = num.sum(axis=-1, keepdims=True) + np.exp(-m)
    return num / den


def softmax1_backward(p: np.ndarray, dy: np.ndarray) -> np.ndarray:
    """Jacobian-vector product of softmax1: dx = p * (dy - sum(p * dy))."""
    return p * (dy - (p * dy).sum(axis=-1, keepdims=True))


def sparsemax_threshold(z: np.ndarray):
    """tau and support size of max-shifted scores (vutils/entmax.py:35-79)."""
    srt = -np.sort(-z, axis=-1)
    with np.errstate(over="ignore", invalid="ignore"):
        cs = np.cumsum(srt, axis=-1) - 1
        rho = _rho(z.shape[-1], z.dtype)
        support = rho * srt > cs
    k = support.sum(axis=-1, keepdims=True)
    tau = np.take_along_axis(cs, k - 1, axis=-1) / k.astype(z.dtype)
    return tau, k


def sparsemax(x: np.ndarray, return_stats: bool = False):
    """sparsemax along the last axis (vutils/entmax.py:136-146)."""
    with np.errstate(over="ignore", invalid="ignore"):
        z = x - x.max(axis=-1, keepdims=True)
    tau, k = sparsemax_threshold(z)
    p = np.maximum(z - tau, 0)
    if return_stats:
        return p, tau, k, z
    return p


def sparsemax_backward(p: np.ndarray, dy: np.ndarray, k: np.ndarray | None = None) -> np.ndarray:
    """SparsemaxFunction.backward (vutils/entmax.py:148-157).

    ``k`` is the support size reported by the threshold search; when omitted
    it is the number of nonzero outputs (they agree unless an entry sits
    exactly on tau).
    """
    nz = p != 0
    if k is None:
        k = nz.sum(axis=-1, keepdims=True)
    g = np.where(nz, dy, 0)
    v_hat = g.sum(axis=-1, keepdims=True) / k.astype(p.dtype)
    return np.where(nz, g - v_hat, g)


def entmax_threshold(z: np.ndarray):
    """tau and support size of halved, max-shifted scores (vutils/entmax.py:82-133)."""
    srt = -np.sort(-z, axis=-1)
    rho = _rho(z.shape[-1], z.dtype)
    with np.errstate(over="ignore", invalid="ignore"):
        mean = np.cumsum(srt, axis=-1) / rho
        mean_sq = np.cumsum(srt * srt, axis=-1) / rho
        ss = rho * (mean_sq - mean * mean)
        delta = (1 - ss) / rho
        delta_nz = np.maximum(delta, 0)
        tau = mean - np.sqrt(delta_nz)
        support = (tau <= srt).sum(axis=-1, keepdims=True)
    tau_star = np.take_along_axis(tau, support - 1, axis=-1)
    return tau_star, support


def entmax15(x: np.ndarray, return_stats: bool = False):
    """1.5-entmax along the last axis (vutils/entmax.py:160-173)."""
    with np.errstate(over="ignore", invalid="ignore"):
        z = (x - x.max(axis=-1, keepdims=True)) / 2
    tau, k = entmax_threshold(z)
    with np.errstate(over="ignore", invalid="ignore"):
        p = np.maximum(z - tau, 0) ** 2
    if return_stats:
        return p, tau, k, z
    return p


def entmax15_backward(p: np.ndarray, dy: np.ndarray) -> np.ndarray:
    """Entmax15Function.backward (vutils/entmax.py:175-183)."""
    g = np.sqrt(p)
    dx = dy * g
    q = dx.sum(axis=-1, keepdims=True) / g.sum(axis=-1, keepdims=True)
    return dx - q * g


def normalize(name: str, x: np.ndarray) -> np.ndarray:
    if name in ("softmax1", "softmax_1"):
        return softmax1(x)
    if name == "sparsemax":
        return sparsemax(x)
    if name == "entmax15":
        return entmax15(x)
    raise ValueError(f"unknown normalizer {name!r}")


def normalize_backward(name: str, x: np.ndarray, p: np.ndarray, dy: np.ndarray) -> np.ndarray:
    if name in ("softmax1", "softmax_1"):
        return softmax1_backward(p, dy)
    if name == "sparsemax":
        _, _, k, _ = sparsemax(x, return_stats=True)
        return sparsemax_backward(p, dy, k)
    if name == "entmax15":
        return entmax15_backward(p, dy)
    raise ValueError(f"unknown normalizer {name!r}")
