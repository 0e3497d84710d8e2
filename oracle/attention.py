"""Attention oracle (dense, varlen, paged) in numpy.  TEST INFRASTRUCTURE.

Restates the reference's eager attention paths:

* dense  -- ``backends.py:44-78`` (``scaled_dot_product_attention``): GQA by
  repeat_interleave, scores = q k^T * scale, masked entries filled with
  ``finfo(dtype).min``, row normalizer, times v.  The causal mask here is the
  one the reference *kernels* use (bottom-right aligned,
  ``kernels/softmax1_hopper.py:79`` ``causal_limit = l + Lk - Lq``); for
  Lq == Lk it equals the eager path's top-left ``tril``.  ``window_left``
  follows ``kernels/softmax1_hopper.py:89-90``.
* varlen -- ``tests/test_varlen_attention.py:10-28`` (``_packed_reference``):
  per-sequence slices of packed [T, H, D] tensors, bottom-right causal.
* paged  -- ``paged.py:184-249`` (``paged_attention``) and
  ``tests/test_paged_attention.py:14-43`` (``_dense_reference``): gather the
  physical tokens ``block_table[b, t // bs] * bs + t % bs`` of each sequence,
  bottom-right causal against the sequence length.

Backward is the analytic chain rule the reference's autograd produces:
dP = dO v^T, dS = normalizer_backward(P, dP), dQ = dS k * scale,
dK = dS^T q * scale, dV = P^T dO, with GQA gradients summed over the group.
"""

from __future__ import annotations

import numpy as np

from .normalizers import normalize, normalize_backward


def _mask(lq: int, lk: int, causal: bool, window_left: int | None):
    qi = np.arange(lq)[:, None]
    kj = np.arange(lk)[None, :]
    valid = np.ones((lq, lk), dtype=bool)
    limit = qi + lk - lq
    if causal:
        valid &= kj <= limit
    if window_left is not None and window_left > 0:
        valid &= kj > limit - window_left
    return valid


def _scores(q, k, scale, valid, dtype):
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    return np.where(valid, s, np.finfo(dtype).min).astype(dtype)


def attention_forward(q, k, v, normalizer, scale=None, causal=True, window_left=None,
                      dtype=np.float64, return_probs=False):
    """q [B,Hq,Lq,D], k/v [B,Hkv,Lk,D] -> o [B,Hq,Lq,D] (numpy, ``dtype``)."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    g = q.shape[1] // k.shape[1]
    if g != 1:
        k = np.repeat(k, g, axis=1)
        v = np.repeat(v, g, axis=1)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    valid = _mask(q.shape[2], k.shape[2], causal, window_left)
    s = _scores(q, k, scale, valid, dtype)
    p = normalize(normalizer, s)
    o = np.matmul(p, v)
    if return_probs:
        return o, p, s
    return o


def attention_backward(q, k, v, do, normalizer, scale=None, causal=True, window_left=None,
                       dtype=np.float64, dropout=None):
    """Returns (o, dq, dk, dv) for upstream gradient ``do``.

    ``dropout = (keep, p)``: keep a bool [B, Hq, Lq, Lk] mask; the output uses
    p_ij keep_ij / (1 - p) and the normalizer's backward receives
    dP keep / (1 - p), as ``kernels/softmax1_hopper.py:105-110, 253-256`` and
    ``kernels/sparse_entmax_hopper.py:141-145, 262-264`` compute them."""
    q = np.asarray(q, dtype=dtype)
    k0 = np.asarray(k, dtype=dtype)
    v0 = np.asarray(v, dtype=dtype)
    do = np.asarray(do, dtype=dtype)
    g = q.shape[1] // k0.shape[1]
    k = np.repeat(k0, g, axis=1) if g != 1 else k0
    v = np.repeat(v0, g, axis=1) if g != 1 else v0
    if scale is None:
        scale = q.shape[-1] ** -0.5
    valid = _mask(q.shape[2], k.shape[2], causal, window_left)
    s = _scores(q, k, scale, valid, dtype)
    p = normalize(normalizer, s)
    factor = 1.0 if dropout is None else np.asarray(dropout[0], dtype=dtype) / (1.0 - float(np.float32(dropout[1])))
    pd = p * factor
    o = np.matmul(pd, v)
    dp = np.matmul(do, np.swapaxes(v, -1, -2)) * factor
    ds = normalize_backward(normalizer, s, p, dp)
    ds = np.where(valid, ds, 0)
    dq = np.matmul(ds, k) * scale
    dk = np.matmul(np.swapaxes(ds, -1, -2), q) * scale
    dv = np.matmul(np.swapaxes(pd, -1, -2), do)
    if g != 1:
        b, h, l, d = dk.shape
        dk = dk.reshape(b, h // g, g, l, d).sum(axis=2)
        dv = dv.reshape(b, h // g, g, l, d).sum(axis=2)
    return o, dq, dk, dv


def _seq_bounds(cu):
    cu = np.asarray(cu, dtype=np.int64)
    return [(int(cu[i]), int(cu[i + 1])) for i in range(len(cu) - 1)]


def varlen_forward(q, k, v, cu_q, cu_k, normalizer, scale=None, causal=True, dtype=np.float64):
    """Packed q [Tq,Hq,D], k/v [Tk,Hkv,D] -> o [Tq,Hq,D]."""
    out = np.zeros(q.shape, dtype=dtype)
    for (q0, q1), (k0, k1) in zip(_seq_bounds(cu_q), _seq_bounds(cu_k)):
        qs = np.swapaxes(np.asarray(q[q0:q1], dtype=dtype), 0, 1)[None]
        ks = np.swapaxes(np.asarray(k[k0:k1], dtype=dtype), 0, 1)[None]
        vs = np.swapaxes(np.asarray(v[k0:k1], dtype=dtype), 0, 1)[None]
        o = attention_forward(qs, ks, vs, normalizer, scale, causal, dtype=dtype)
        out[q0:q1] = np.swapaxes(o[0], 0, 1)
    return out


def varlen_backward(q, k, v, do, cu_q, cu_k, normalizer, scale=None, causal=True, dtype=np.float64):
    o = np.zeros(q.shape, dtype=dtype)
    dq = np.zeros(q.shape, dtype=dtype)
    dk = np.zeros(k.shape, dtype=dtype)
    dv = np.zeros(v.shape, dtype=dtype)
    for (q0, q1), (k0, k1) in zip(_seq_bounds(cu_q), _seq_bounds(cu_k)):
        t = lambda a, s, e: np.swapaxes(np.asarray(a[s:e], dtype=dtype), 0, 1)[None]  # noqa: E731
        r = attention_backward(t(q, q0, q1), t(k, k0, k1), t(v, k0, k1), t(do, q0, q1),
                               normalizer, scale, causal, dtype=dtype)
        o[q0:q1] = np.swapaxes(r[0][0], 0, 1)
        dq[q0:q1] = np.swapaxes(r[1][0], 0, 1)
        dk[k0:k1] = np.swapaxes(r[2][0], 0, 1)
        dv[k0:k1] = np.swapaxes(r[3][0], 0, 1)
    return o, dq, dk, dv


def _physical(block_table, b, length, block_size):
    pos = np.arange(length)
    return np.asarray(block_table)[b, pos // block_size].astype(np.int64) * block_size + pos % block_size


def paged_forward(q, key_cache, value_cache, block_table, seq_lens, block_size, normalizer,
                  scale=None, causal=True, dtype=np.float64):
    """q [B,Hq,Lq,D]; caches [P*bs,Hkv,D]; returns o [B,Hq,Lq,D]."""
    out = np.zeros(q.shape, dtype=dtype)
    for b, length in enumerate(np.asarray(seq_lens).tolist()):
        phys = _physical(block_table, b, length, block_size)
        ks = np.swapaxes(np.asarray(key_cache[phys], dtype=dtype), 0, 1)[None]
        vs = np.swapaxes(np.asarray(value_cache[phys], dtype=dtype), 0, 1)[None]
        out[b] = attention_forward(np.asarray(q[b:b + 1], dtype=dtype), ks, vs, normalizer,
                                   scale, causal, dtype=dtype)[0]
    return out


def paged_backward(q, key_cache, value_cache, do, block_table, seq_lens, block_size, normalizer,
                   scale=None, causal=True, dtype=np.float64):
    """Returns (o, dq, dkey_cache, dvalue_cache); cache grads scatter-add into pages."""
    o = np.zeros(q.shape, dtype=dtype)
    dq = np.zeros(q.shape, dtype=dtype)
    dkc = np.zeros(key_cache.shape, dtype=dtype)
    dvc = np.zeros(value_cache.shape, dtype=dtype)
    for b, length in enumerate(np.asarray(seq_lens).tolist()):
        phys = _physical(block_table, b, length, block_size)
        ks = np.swapaxes(np.asarray(key_cache[phys], dtype=dtype), 0, 1)[None]
        vs = np.swapaxes(np.asarray(value_cache[phys], dtype=dtype), 0, 1)[None]
        r = attention_backward(np.asarray(q[b:b + 1], dtype=dtype), ks, vs,
                               np.asarray(do[b:b + 1], dtype=dtype), normalizer, scale, causal,
                               dtype=dtype)
        o[b] = r[0][0]
        dq[b] = r[1][0]
        np.add.at(dkc, phys, np.swapaxes(r[2][0], 0, 1))
        np.add.at(dvc, phys, np.swapaxes(r[3][0], 0, 1))
    return o, dq, dkc, dvc
