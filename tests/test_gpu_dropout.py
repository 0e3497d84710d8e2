"""Fused attention dropout on the tensor-core kernels (16-bit inputs, head_dim
64 / 128), against the oracle run with the very keep mask the kernels draw.

The kernels regenerate the mask from a saved device seed with a counter-based
generator (Philox4x32-10); ``oracle.philox`` restates the same counter layout,
so the oracle can apply the identical mask: o = (p keep / (1 - p_drop)) V and
the normalizer backward receives dP keep / (1 - p_drop).  The reference's own
test of this feature (tests/test_hopper_attention.py:75-98) checks that two
runs after the same torch.manual_seed are bit-identical with finite
gradients; that check is here too.
"""

import numpy as np
import pytest
import torch

import oracle
from hf_attention_normalizers_b200 import _native as N
from hf_attention_normalizers_b200 import kernels, ops

from test_gpu_parity import _inputs, _np, assert_close

pytestmark = pytest.mark.gpu

NORMS = ("softmax1", "sparsemax", "entmax15")
KERNELS = {
    "softmax1": kernels.hopper_softmax1_attention,
    "sparsemax": kernels.hopper_sparsemax_attention,
    "entmax15": kernels.hopper_entmax15_attention,
}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", [(2, 4, 2, 200, 64), (1, 8, 2, 300, 128)])
@pytest.mark.parametrize("norm", NORMS)
def test_dropout_matches_oracle_with_the_same_mask(norm, case, dtype):
    b, hq, hkv, s, d = case
    p_drop, seed_value = 0.3, 123456789
    q, k, v, do = _inputs((b, hq, s, d), (b, hkv, s, d), dtype, seed=7 + d)
    seed = torch.tensor(seed_value, dtype=torch.int64, device="cuda")
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = ops.attn_fwd(qr, kr, vr, N.NORMALIZER_IDS[norm], d ** -0.5, True, -1, False, p_drop, seed)[0]
    o.backward(do)
    torch.cuda.synchronize()
    keep = oracle.philox.keep_mask(seed_value, p_drop, b, hq, s, s)
    assert abs(keep.mean() - (1 - p_drop)) < 0.01
    ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), norm, causal=True, dropout=(keep, p_drop))
    for label, a, e in zip(("o", "dq", "dk", "dv"), (o, qr.grad, kr.grad, vr.grad), ref):
        assert_close(a, e, dtype, f"dropout/{norm}/{case}/{label}")


@pytest.mark.parametrize("norm", NORMS)
def test_fused_dropout_is_reproducible_and_has_finite_backward(norm):
    """tests/test_hopper_attention.py:75-98 at a tensor-core shape: the same
    torch seed gives bit-identical outputs and gradients; another seed gives
    another mask."""
    torch.manual_seed(41)
    inputs = [torch.randn(1, 2, 177, 64, device="cuda", dtype=torch.float16) for _ in range(3)]
    runs = []
    for torch_seed in (97, 97, 98):
        q, k, v = (t.detach().clone().requires_grad_(True) for t in inputs)
        torch.manual_seed(torch_seed)
        out = KERNELS[norm](q, k, v, is_causal=True, dropout_p=0.2)
        out.float().square().mean().backward()
        runs.append((out.detach(), q.grad, k.grad, v.grad))
    for a, b in zip(runs[0], runs[1]):
        assert torch.equal(a, b)
        assert torch.isfinite(a).all()
    assert not torch.equal(runs[0][0], runs[2][0])


def test_dropout_on_unsupported_inputs_raises():
    q = torch.randn(1, 2, 16, 32, device="cuda")
    with pytest.raises(NotImplementedError, match="dropout"):
        kernels.hopper_softmax1_attention(q, q, q, is_causal=True, dropout_p=0.1)
