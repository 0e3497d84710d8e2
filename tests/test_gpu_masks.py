"""Masks the fused kernels run without materialising scores: HF's causal mask
of a right-padded batch (one launch, per-sequence key counts, causal mask
aligned at the first key), sliding windows and pure causal masks, given as
HF 4-D boolean / additive masks or as Flex BlockMasks.  Reference routes:
backends.py:183-568 (right-padded Hopper attention, causal / sliding
BlockMasks)."""

import numpy as np
import pytest
import torch

import oracle
from hf_attention_normalizers_b200 import backends, ops
from hf_attention_normalizers_b200 import _native as N

from test_gpu_parity import _inputs, _np, assert_close

pytestmark = pytest.mark.gpu

NORMS = ("softmax1", "sparsemax", "entmax15")


def _padded_reference(norm, q, k, v, do, lengths):
    """Row i of sequence b sees keys j <= i, j < lengths[b]: causal over the
    valid prefix, and the padded query rows see the whole prefix (the split
    of backends.py:447-470)."""
    outs = [np.zeros(q.shape) for _ in range(2)] + [np.zeros(k.shape) for _ in range(2)]
    for b, length in enumerate(lengths):
        qb, dob, kb, vb = q[b:b + 1], do[b:b + 1], k[b:b + 1, :, :length], v[b:b + 1, :, :length]
        if length == 0:
            continue
        r = oracle.attention_backward(qb[:, :, :length], kb, vb, dob[:, :, :length], norm, causal=True)
        outs[0][b, :, :length], outs[1][b, :, :length] = r[0][0], r[1][0]
        outs[2][b, :, :length] += r[2][0]
        outs[3][b, :, :length] += r[3][0]
        if length < q.shape[2]:
            r = oracle.attention_backward(qb[:, :, length:], kb, vb, dob[:, :, length:], norm, causal=False)
            outs[0][b, :, length:], outs[1][b, :, length:] = r[0][0], r[1][0]
            outs[2][b, :, :length] += r[2][0]
            outs[3][b, :, :length] += r[3][0]
    return outs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("norm", NORMS)
def test_key_lengths_right_padded_batch_matches_oracle(norm, dtype):
    b, hq, hkv, s, d = 3, 4, 2, 260, 128
    lengths = [260, 131, 7]
    q, k, v, do = _inputs((b, hq, s, d), (b, hkv, s, d), dtype, seed=17)
    kl = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = ops.attn_fwd(qr, kr, vr, N.NORMALIZER_IDS[norm], d ** -0.5, True, -1, False, 0.0, None, kl)[0]
    o.backward(do)
    ref = _padded_reference(norm, _np(q), _np(k), _np(v), _np(do), lengths)
    for label, a, e in zip(("o", "dq", "dk", "dv"), (o, qr.grad, kr.grad, vr.grad), ref):
        assert_close(a, e, dtype, f"padded/{norm}/{label}")


def _hf_mask(lengths, s, additive, dtype=torch.float32):
    i = torch.arange(s, device="cuda")[:, None]
    j = torch.arange(s, device="cuda")[None, :]
    allowed = (j <= i)[None] & (j[None] < torch.tensor(lengths, device="cuda")[:, None, None])
    allowed = allowed[:, None]
    if not additive:
        return allowed
    return torch.zeros(allowed.shape, dtype=dtype, device="cuda").masked_fill(~allowed, torch.finfo(dtype).min)


class _Module(torch.nn.Module):
    is_causal = True
    num_key_value_groups = 2


@pytest.mark.parametrize("additive", [False, True])
@pytest.mark.parametrize("norm", NORMS)
def test_hf_padding_mask_runs_fused_and_matches_materialised(norm, additive, monkeypatch):
    b, hq, hkv, s, d = 2, 4, 2, 200, 128
    q, k, v, _ = _inputs((b, hq, s, d), (b, hkv, s, d), torch.bfloat16, seed=23)
    lengths = [200, 150]
    mask = _hf_mask(lengths, s, additive, torch.bfloat16)
    calls = []
    real = ops.attn_fwd
    monkeypatch.setattr(ops, "attn_fwd", lambda *a, **kw: calls.append(a[-1] if len(a) > 10 else None) or real(*a, **kw))
    fn = {"softmax1": backends.softmax_1, "sparsemax": backends.sparsemax, "entmax15": backends.entmax15}[norm]
    fused, _ = backends.sdpa_attention_forward(_Module().eval(), q, k, v, mask, softmax_fn=fn, scaling=d ** -0.5)
    assert len(calls) == 1 and calls[0] is not None, "the padded mask did not take the fused route"
    ref = _padded_reference(norm, _np(q), _np(k), _np(v), _np(q), lengths)[0]
    assert_close(fused.transpose(1, 2), ref, torch.bfloat16, f"hf padding/{norm}")


@pytest.mark.parametrize("norm", NORMS)
def test_flex_block_masks_route_to_fused_kernel(norm, monkeypatch):
    from torch.nn.attention.flex_attention import create_block_mask

    b, hq, hkv, s, d, w = 2, 4, 2, 256, 128, 40
    q, k, v, _ = _inputs((b, hq, s, d), (b, hkv, s, d), torch.bfloat16, seed=29)
    lengths = torch.tensor([256, 100], device="cuda")
    fn = {"softmax1": backends.softmax_1, "sparsemax": backends.sparsemax, "entmax15": backends.entmax15}[norm]
    launched = []
    real = ops.attn_fwd
    monkeypatch.setattr(ops, "attn_fwd", lambda *a, **kw: launched.append(a) or real(*a, **kw))
    cases = {
        "causal": lambda bb, h, qi, ki: ki <= qi,
        "window": lambda bb, h, qi, ki: (ki <= qi) & (ki > qi - w),
        "padded": lambda bb, h, qi, ki: (ki <= qi) & (ki < lengths[bb]),
    }
    for label, mod in cases.items():
        launched.clear()
        bm = create_block_mask(mod, b, None, s, s, device="cuda")
        out, _ = backends.flex_attention_normalizer_forward(_Module().eval(), q, k, v, bm, softmax_fn=fn,
                                                            scaling=d ** -0.5)
        assert len(launched) == 1, f"{label}: not the fused route"
        if label == "causal":
            ref = oracle.attention_forward(_np(q), _np(k), _np(v), norm, causal=True)
        elif label == "window":
            ref = oracle.attention_forward(_np(q), _np(k), _np(v), norm, causal=True, window_left=w)
        else:
            ref = _padded_reference(norm, _np(q), _np(k), _np(v), _np(q), lengths.tolist())[0]
        assert_close(out.transpose(1, 2), ref, torch.bfloat16, f"flex/{label}/{norm}")
