"""Dropout keep mask of the fused kernels, in numpy.  TEST INFRASTRUCTURE.

The reference draws its dropout mask with Triton's counter-based tl.rand
(``kernels/softmax1_hopper.py:105-110``, ``kernels/sparse_entmax_hopper.py:141-145``):
keep = uniform(seed, offset) >= p, regenerated in the backward from the saved
seed.  The engine does the same with its own counter layout over the
Philox4x32-10 generator (Salmon, Moraes, Dror and Shaw, SC 2011), restated
here so that tests can rebuild the exact mask a kernel used:

  element (row r = (b * heads_q + h) * len_q + i, key j):
  counter (j // 4, r & 0xffffffff, r >> 32, 0), key (seed & 0xffffffff, seed >> 32),
  word j % 4, keep = (word >> 8) >= ceil(p * 2**24).
"""

from __future__ import annotations

import math

import numpy as np

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    c0, c1, c2, c3 = (np.asarray(x, dtype=np.uint32) for x in (c0, c1, c2, c3))
    k0, k1 = np.uint32(k0), np.uint32(k1)
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * c0.astype(np.uint64)
            p1 = _M1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & _MASK32).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & _MASK32).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            k0 = np.uint32(k0 + _W0)
            k1 = np.uint32(k1 + _W1)
    return c0, c1, c2, c3


def keep_mask(seed: int, p: float, batch: int, heads: int, len_q: int, len_k: int) -> np.ndarray:
    """bool [batch, heads, len_q, len_k]: True where the element is kept."""
    thr = max(1, math.ceil(float(np.float32(p)) * 2 ** 24))  # the kernels get p as float32
    r = np.arange(batch * heads * len_q, dtype=np.uint64)[:, None]
    g = np.arange((len_k + 3) // 4, dtype=np.uint64)[None, :]
    r, g = np.broadcast_arrays(r, g)
    words = philox4x32_10(g, r & _MASK32, r >> np.uint64(32), np.zeros_like(g), seed & 0xFFFFFFFF, seed >> 32)
    w = np.stack(words, axis=-1).reshape(batch * heads * len_q, -1)[:, :len_k]
    return ((w >> np.uint32(8)) >= thr).reshape(batch, heads, len_q, len_k)
