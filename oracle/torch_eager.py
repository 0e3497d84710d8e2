"""The reference's eager attention path restated with torch CPU ops.  TEST INFRASTRUCTURE.

The reference package cannot be imported where the benchmarks run, so the
CPU baseline times this restatement instead: the same torch operations the
reference's eager path executes, on the host cores, float32.

* attention -- ``hf_attention_normalizers/backends.py:44-78``
  (``scaled_dot_product_attention``): scores = q k^T * scale, masked entries
  filled with ``finfo.min``, row normalizer, times v.  GQA is handled by
  broadcasting one KV head against its group of query heads (the reference
  repeats K and V; the products are the same).
* normalizers -- ``vutils/softmax1.py:4-28`` (max shift, exp, denominator
  plus exp(-max)); ``vutils/entmax.py:35-79, 136-157`` (sparsemax: full
  descending sort, cumsum, support test, tau, closed-form backward);
  ``vutils/entmax.py:82-133, 160-183`` (1.5-entmax: halved scores, sorted
  running mean and mean of squares, tau, closed-form backward without the
  1/2 of the rescaling, as the reference computes it).
* backward -- the chain rule the reference's autograd runs: dP = dO v^T,
  dS from the normalizer's closed form, dQ = dS k scale, dK = dS^T q scale,
  dV = P^T dO.

The numbers match ``oracle.attention_backward`` (numpy, pinned to the
reference's golden vectors) to rounding; ``tests/test_oracle.py`` checks it.
"""

from __future__ import annotations

import torch


def _softmax1(x):
    m = x.amax(dim=-1, keepdim=True)
    num = torch.exp(x - m)
    return num / (num.sum(dim=-1, keepdim=True) + torch.exp(-m))


def _rho(n, like):
    return torch.arange(1, n + 1, dtype=like.dtype, device=like.device)


def _sparsemax(x):
    z = x - x.amax(dim=-1, keepdim=True)
    srt, _ = torch.sort(z, dim=-1, descending=True)
    cs = srt.cumsum(dim=-1) - 1
    k = (_rho(z.shape[-1], z) * srt > cs).sum(dim=-1, keepdim=True)
    tau = cs.gather(-1, k - 1) / k.to(z.dtype)
    return torch.clamp(z - tau, min=0), k


def _entmax15(x):
    z = (x - x.amax(dim=-1, keepdim=True)) / 2
    srt, _ = torch.sort(z, dim=-1, descending=True)
    rho = _rho(z.shape[-1], z)
    mean = srt.cumsum(dim=-1) / rho
    mean_sq = (srt * srt).cumsum(dim=-1) / rho
    delta = (1 - rho * (mean_sq - mean * mean)) / rho
    tau = mean - torch.sqrt(torch.clamp(delta, min=0))
    k = (tau <= srt).sum(dim=-1, keepdim=True)
    tau_star = tau.gather(-1, k - 1)
    return torch.clamp(z - tau_star, min=0) ** 2


def attention_backward(q, k, v, do, normalizer, scale=None, causal=True):
    """q, do [B, Hq, Lq, D]; k, v [B, Hkv, Lk, D] (torch CPU tensors).
    Returns (o, dq, dk, dv); causal masks are bottom-right aligned."""
    b, hq, lq, d = q.shape
    hkv, lk = k.shape[1], k.shape[2]
    g = hq // hkv
    if scale is None:
        scale = d ** -0.5
    qg = q.reshape(b, hkv, g, lq, d)
    dog = do.reshape(b, hkv, g, lq, d)
    kk, vv = k.unsqueeze(2), v.unsqueeze(2)
    s = qg @ kk.transpose(-1, -2) * scale
    if causal:
        qi = torch.arange(lq).unsqueeze(1)
        kj = torch.arange(lk).unsqueeze(0)
        valid = kj <= qi + (lk - lq)
        s = s.masked_fill(~valid, torch.finfo(s.dtype).min)
    if normalizer in ("softmax1", "softmax_1"):
        p = _softmax1(s)
    elif normalizer == "sparsemax":
        p, ksup = _sparsemax(s)
    elif normalizer == "entmax15":
        p = _entmax15(s)
    else:
        raise ValueError(f"unknown normalizer {normalizer!r}")
    o = p @ vv
    dp = dog @ vv.transpose(-1, -2)
    if normalizer in ("softmax1", "softmax_1"):
        ds = p * (dp - (p * dp).sum(dim=-1, keepdim=True))
    elif normalizer == "sparsemax":
        nz = p != 0
        gsum = torch.where(nz, dp, 0).sum(dim=-1, keepdim=True)
        ds = torch.where(nz, dp - gsum / ksup.to(dp.dtype), 0)
    else:
        w = torch.sqrt(p)
        dx = dp * w
        ds = dx - (dx.sum(dim=-1, keepdim=True) / w.sum(dim=-1, keepdim=True)) * w
    if causal:
        ds = ds.masked_fill(~valid, 0)
    dq = (ds @ kk) * scale
    dk = (ds.transpose(-1, -2) @ qg).sum(dim=2) * scale
    dv = (p.transpose(-1, -2) @ dog).sum(dim=2)
    return (o.reshape(b, hq, lq, d), dq.reshape(b, hq, lq, d), dk, dv)
