"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which ran the
reference's eager code (vutils normalizers, ``backends.scaled_dot_product_attention``,
``paged.paged_attention`` and the varlen test loop) on the reference tests'
own seeds.  Tolerances: float64 cases agree to 1e-10; float32 normalizer
cases to 1e-6 (both implementations sort and cumsum in float32).
"""

import numpy as np
import pytest
import torch

import oracle

NORMS = ("softmax1", "sparsemax", "entmax15")


@pytest.mark.parametrize("label", ["plain", "masked"])
@pytest.mark.parametrize("dt", ["f64", "f32"])
@pytest.mark.parametrize("name", NORMS)
def test_normalizers_match_reference(golden, name, dt, label):
    g = golden("normalizers")
    x = g[f"norm_{label}_{dt}_x"]
    dy = g[f"norm_{label}_{dt}_dy"]
    y = oracle.normalize(name, x)
    dx = oracle.normalize_backward(name, x, y, dy)
    tol = 1e-10 if dt == "f64" else 2e-6
    np.testing.assert_allclose(y, g[f"norm_{label}_{dt}_{name}_y"], rtol=0, atol=tol)
    np.testing.assert_allclose(dx, g[f"norm_{label}_{dt}_{name}_dx"], rtol=0, atol=tol * 10)


@pytest.mark.parametrize("tag", ["mha", "gqa"])
@pytest.mark.parametrize("name", NORMS)
def test_dense_attention_matches_reference(golden, tag, name):
    g = golden("dense")
    q, k, v, do = (g[f"dense_{tag}_{x}"] for x in ("q", "k", "v", "do"))
    o, dq, dk, dv = oracle.attention_backward(q, k, v, do, name, causal=True)
    for label, a in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(a, g[f"dense_{tag}_{name}_{label}"], rtol=0, atol=1e-10)


@pytest.mark.parametrize("name", NORMS)
def test_varlen_matches_reference_loop(golden, name):
    g = golden("varlen")
    q, k, v, do = (g[f"varlen_{name}_{x}"] for x in ("q", "k", "v", "do"))
    o, dq, dk, dv = oracle.varlen_backward(q, k, v, do, g["varlen_cu_q"], g["varlen_cu_k"], name)
    for label, a in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(a, g[f"varlen_{name}_{label}"], rtol=0, atol=1e-10)


@pytest.mark.parametrize("tag", ["unique", "shared", "decode"])
@pytest.mark.parametrize("name", NORMS)
def test_paged_matches_reference(golden, tag, name):
    g = golden("paged")
    pre = f"paged_{tag}_{name}_"
    o, dq, dkc, dvc = oracle.paged_backward(
        g[pre + "q"], g[pre + "kc"], g[pre + "vc"], g[pre + "do"], g[f"paged_{tag}_block_table"],
        g[f"paged_{tag}_seq_lens"], int(g[f"paged_{tag}_block_size"]), name)
    for label, a in (("o", o), ("dq", dq), ("dkc", dkc), ("dvc", dvc)):
        np.testing.assert_allclose(a, g[pre + label], rtol=0, atol=1e-10)


@pytest.mark.parametrize("name", NORMS)
def test_config1_fp32_matches_reference(golden, name):
    """BASELINE config 1 in float32 on the reference's seed; sampled rows + sums."""
    g = golden("config1")
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 8, 512, 128) for _ in range(3))
    o_shape = q.shape
    gr = torch.randn(o_shape)
    o, dq, dk, dv = oracle.attention_backward(q.numpy(), k.numpy(), v.numpy(), gr.numpy(), name,
                                              scale=1 / np.sqrt(128), causal=True, dtype=np.float32)
    for label, a in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        ref = g[f"config1_{name}_{label}_rows"]
        np.testing.assert_allclose(a[:, :, ::61, :], ref, rtol=0, atol=2e-5)
        assert abs(a.astype(np.float64).sum() - float(g[f"config1_{name}_{label}_sum"])) < 1e-2


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors (Random123's kat_vectors, as
    published with the generator): counter/key all zeros and all ones."""
    from oracle import philox

    assert [int(x) for x in philox.philox4x32_10(0, 0, 0, 0, 0, 0)] == [
        0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    ones = 0xFFFFFFFF
    assert [int(x) for x in philox.philox4x32_10(ones, ones, ones, ones, ones, ones)] == [
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]


def test_dropout_keep_rate_and_oracle_identity():
    import numpy as np

    from oracle import philox
    import oracle

    keep = philox.keep_mask(7, 0.25, 2, 3, 64, 96)
    assert abs(keep.mean() - 0.75) < 0.02
    assert not np.array_equal(keep, philox.keep_mask(8, 0.25, 2, 3, 64, 96))
    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((1, 2, 16, 8)) for _ in range(4))
    base = oracle.attention_backward(q, k, v, do, "entmax15")
    all_kept = oracle.attention_backward(q, k, v, do, "entmax15", dropout=(np.ones((1, 2, 16, 16), bool), 0.0))
    for a, b in zip(base, all_kept):
        assert np.allclose(a, b, rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", ["softmax1", "sparsemax", "entmax15"])
@pytest.mark.parametrize("hq,hkv,lq,lk", [(4, 4, 64, 64), (8, 2, 48, 96)])
def test_torch_eager_restatement_matches_oracle(name, hq, hkv, lq, lk):
    """The CPU baseline's torch restatement of the reference's eager path
    computes what the pinned numpy oracle computes (float64, both causal)."""
    from oracle import torch_eager

    rng = np.random.default_rng(7)
    q = rng.standard_normal((2, hq, lq, 32))
    k = rng.standard_normal((2, hkv, lk, 32))
    v = rng.standard_normal((2, hkv, lk, 32))
    do = rng.standard_normal((2, hq, lq, 32))
    ref = oracle.attention_backward(q, k, v, do, name, causal=True)
    got = torch_eager.attention_backward(*(torch.from_numpy(x) for x in (q, k, v, do)), name, causal=True)
    for label, a, e in zip(("o", "dq", "dk", "dv"), got, ref):
        assert np.abs(a.numpy() - e).max() <= 1e-10 * max(1.0, np.abs(e).max()), label


@pytest.mark.parametrize("name", NORMS)
def test_torch_eager_config1_matches_reference(golden, name):
    """BASELINE config 1 (float32, the reference's seed) through the torch
    restatement, against the reference's own sampled rows and sums."""
    from oracle import torch_eager

    g = golden("config1")
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 8, 512, 128) for _ in range(3))
    gr = torch.randn(q.shape)
    got = torch_eager.attention_backward(q, k, v, gr, name, scale=1 / np.sqrt(128), causal=True)
    for label, a in zip(("o", "dq", "dk", "dv"), got):
        a = a.numpy()
        np.testing.assert_allclose(a[:, :, ::61, :], g[f"config1_{name}_{label}_rows"], rtol=0, atol=2e-5)
        assert abs(a.astype(np.float64).sum() - float(g[f"config1_{name}_{label}_sum"])) < 1e-2
