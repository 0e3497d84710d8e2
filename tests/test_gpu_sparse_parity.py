"""GPU parity of the tensor-core sparse path (bf16 / fp16 inputs) against the
numpy oracle, at the BASELINE shapes and on the wide-support route.

What is checked, beyond outputs and gradients:
  * the saved threshold tau (stats[0], z units) against the oracle's sort-based
    tau of vutils/entmax.py:35-133, within TAU_TOL (1 + |tau|);
  * the zero pattern: the saved support size (stats[1]) equals the oracle's
    count of z > tau on every row that has no score within NEAR of tau.
    The kernel's scores are fp32 tensor-core dot products of the 16-bit
    inputs; the oracle's are float64 dot products of the same values.  For
    D = 128 and scores of order ten the two differ by a few 1e-6 (fp32
    accumulation over 128 products), so entries closer to tau than NEAR can
    fall on either side; that bound replaces the 1e-6 of an exact-arithmetic
    comparison.

Long rows are checked on their last R query rows (o, dq, tau, support) and on
their last R keys (dk, dv): under the causal mask only the last R query rows
see those keys, so the oracle runs on an R x Lk slice.
"""

import numpy as np
import pytest
import torch

import oracle
from hf_attention_normalizers_b200 import _native as N
from hf_attention_normalizers_b200 import kernels, ops, varlen

from test_gpu_parity import DENSE_CASES, _inputs, _np, assert_close

pytestmark = pytest.mark.gpu

SPARSE = ("sparsemax", "entmax15")
KERNELS = {
    "softmax1": kernels.hopper_softmax1_attention,
    "sparsemax": kernels.hopper_sparsemax_attention,
    "entmax15": kernels.hopper_entmax15_attention,
}
TAU_TOL = 5e-6
NEAR = 1e-4


def _oracle_threshold(norm, q, k, scale):
    """tau (z units, absolute) and the scores z of every row: q [B,Hq,R,D], k [B,Hkv,Lk,D]
    with the R query rows bottom-right aligned against the Lk keys."""
    _, p, s = oracle.attention_forward(q, k, k, norm, scale=scale, causal=True, return_probs=True)
    half = 1.0 if norm == "sparsemax" else 0.5
    with np.errstate(all="ignore"):
        z = (s - s.max(-1, keepdims=True)) * half
        fn = oracle.normalizers.sparsemax_threshold if norm == "sparsemax" else oracle.normalizers.entmax_threshold
        tau_rel, _ = fn(z)
    tau = tau_rel[..., 0] + s.max(-1) * half
    valid = s > np.finfo(np.float64).min
    return tau, np.where(valid, s * half, -np.inf)


def check_threshold(norm, tau_k, support_k, q, k, scale, what, near=NEAR):
    """tau_k / support_k [B,Hq,R] from the kernel's stats; q the same R rows."""
    tau, z = _oracle_threshold(norm, q, k, scale)
    err = np.abs(tau_k - tau)
    assert np.all(err <= TAU_TOL * (1 + np.abs(tau))), f"{what}: tau max err {err.max():.3e}"
    count = (z > tau[..., None]).sum(-1)
    clean = ~(np.abs(z - tau[..., None]) < near).any(-1)
    bad = (support_k != count) & clean
    assert clean.mean() > 0.5, f"{what}: too few rows without a score near tau ({clean.mean():.2f})"
    assert not bad.any(), f"{what}: support differs on {int(bad.sum())} clean rows"
    return float(err.max()), int(count.max())


def _stats(norm, q, k, v, scale):
    _, st, _, _, _ = ops.attn_fwd(q, k, v, N.NORMALIZER_IDS[norm], scale, True, -1, False)
    b, hq, lq, _ = q.shape  # stats [2][Hq][B * Lq]
    return st.reshape(2, hq, b, lq).transpose(1, 2).double().cpu().numpy()


def _tail_check(norm, q, k, v, do, out, rows, dtype, what, scale=None):
    """o, dq of the last `rows` query rows and dk, dv of the last `rows` keys
    against the oracle (Lq == Lk, causal)."""
    qt, dot = q[:, :, -rows:], do[:, :, -rows:]
    ref = oracle.attention_backward(_np(qt), _np(k), _np(v), _np(dot), norm, scale=scale, causal=True)
    o, dq, dk, dv = out
    assert_close(o[:, :, -rows:], ref[0], dtype, f"{what}/o")
    assert_close(dq[:, :, -rows:], ref[1], dtype, f"{what}/dq")
    assert_close(dk[:, :, -rows:], ref[2][:, :, -rows:], dtype, f"{what}/dk")
    assert_close(dv[:, :, -rows:], ref[3][:, :, -rows:], dtype, f"{what}/dv")


def _fwd_bwd(norm, q, k, v, do, scale=None):
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = KERNELS[norm](qr, kr, vr, scale=scale, is_causal=True)
    o.backward(do)
    torch.cuda.synchronize()
    return o.detach(), qr.grad, kr.grad, vr.grad


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", [c for c in DENSE_CASES if c[5] in (64, 128)])
@pytest.mark.parametrize("norm", SPARSE)
def test_tensor_core_threshold_and_zero_pattern(norm, case, dtype):
    """The tensor-core forward's tau and support size on the random dense cases."""
    b, hq, hkv, lq, lk, d, causal = case
    if not causal:
        pytest.skip("the bottom-right threshold helper assumes a causal mask")
    q, k, v, _ = _inputs((b, hq, lq, d), (b, hkv, lk, d), dtype, seed=100 + DENSE_CASES.index(case))
    st = _stats(norm, q, k, v, d ** -0.5)
    err, _ = check_threshold(norm, st[0], st[1], _np(q), _np(k), d ** -0.5, f"{norm}/{case}/{dtype}")
    print(f"{norm} {case} {dtype}: tau max err {err:.2e}")


@pytest.mark.parametrize("norm", SPARSE)
def test_config2_slice_at_full_length(norm):
    """BASELINE config 2 at its own row length: one (batch, KV group) slice,
    4 query heads on 1 KV head, S = 8192, bf16, q,k,v ~ N(0,1), scale 1/sqrt(128)."""
    rows = 512
    q, k, v, do = _inputs((1, 4, 8192, 128), (1, 1, 8192, 128), torch.bfloat16, seed=2)
    out = _fwd_bwd(norm, q, k, v, do)
    _tail_check(norm, q, k, v, do, out, rows, torch.bfloat16, f"config2/{norm}")
    st = _stats(norm, q, k, v, 128 ** -0.5)
    err, _ = check_threshold(norm, st[0][..., -rows:], st[1][..., -rows:], _np(q[:, :, -rows:]), _np(k),
                             128 ** -0.5, f"config2/{norm}")
    print(f"config2 {norm}: tau max err {err:.2e}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("norm", SPARSE)
def test_wide_support_rows_settled_by_sweeps(norm, dtype):
    """q and k pre-scaled by D^-1/4 (scores ~ N(0, 1/128) after the softmax
    scale; sparsemax another factor 0.3 on each, scores ~ N(0, 1/1400)):
    supports of hundreds of keys (sparsemax) to most of the row (entmax15).
    Rows whose live candidates outgrow the 192-entry buffers are settled by
    exact sweeps over the row; the oracle's support sizes show that such rows
    are present (more than 192 keys), so this case runs that route."""
    rows = 256
    extra = 0.3 if norm == "sparsemax" else 1.0
    q, k, v, do = _inputs((1, 4, 8192, 128), (1, 1, 8192, 128), torch.float32, seed=5)
    q, k = q * (extra * 128 ** -0.25), k * (extra * 128 ** -0.25)
    q, k, v, do = (t.to(dtype) for t in (q, k, v, do))
    out = _fwd_bwd(norm, q, k, v, do)
    _tail_check(norm, q, k, v, do, out, rows, dtype, f"wide/{norm}")
    st = _stats(norm, q, k, v, 128 ** -0.5)
    # scores of order 0.1 (0.03): the fp32 dot products are accurate to ~1e-7
    # (1e-8) here, and the near-tau exclusion shrinks with them (wide
    # supports crowd tau)
    err, top = check_threshold(norm, st[0][..., -rows:], st[1][..., -rows:], _np(q[:, :, -rows:]), _np(k),
                               128 ** -0.5, f"wide/{norm}", near=2e-6 * extra ** 2)
    assert top > 192, f"the case no longer reaches the sweep route (largest support {top})"
    print(f"wide {norm} {dtype}: tau max err {err:.2e}, largest support {top}")


def _config3_lengths():
    return torch.randint(128, 4097, (64,), generator=torch.Generator().manual_seed(0))


@pytest.mark.parametrize("norm", ["softmax1", "sparsemax", "entmax15"])
def test_config3_varlen_seed0_lengths(norm):
    """64 packed sequences with the seed-0 lengths (142,014
    tokens, longest 4095), 16 query heads on 8 KV heads, bf16, causal.  The
    three shortest sequences are compared whole, the longest on its last 256
    query rows and keys."""
    lens = _config3_lengths()
    assert int(lens.sum()) == 142014 and int(lens.max()) == 4095
    cu = torch.zeros(65, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    total = int(cu[-1])
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(total, 16, 128, generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn(total, 8, 128, generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn(total, 8, 128, generator=gen).to(torch.bfloat16).cuda()
    do = torch.randn(total, 16, 128, generator=gen).to(torch.bfloat16).cuda()
    cu_d = cu.cuda()
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = varlen.varlen_hopper_attention(qr, kr, vr, cu_d, cu_d, norm, max_seqlen_q=4095, max_seqlen_k=4095)
    o.backward(do)
    torch.cuda.synchronize()
    out = (o.detach(), qr.grad, kr.grad, vr.grad)

    def seq(t, i):  # packed [T, H, D] -> [1, H, L, D] of sequence i
        return t[int(cu[i]):int(cu[i + 1])].transpose(0, 1).unsqueeze(0)

    order = torch.argsort(lens)
    for i in order[:3].tolist():
        ref = oracle.attention_backward(_np(seq(q, i)), _np(seq(k, i)), _np(seq(v, i)), _np(seq(do, i)), norm,
                                        causal=True)
        for label, a, e in zip(("o", "dq", "dk", "dv"), out, ref):
            assert_close(seq(a, i), e, torch.bfloat16, f"config3/{norm}/seq {i}/{label}")
    i = int(order[-1])
    _tail_check(norm, seq(q, i), seq(k, i), seq(v, i), seq(do, i), tuple(seq(t, i) for t in out), 256,
                torch.bfloat16, f"config3/{norm}/seq {i}")


@pytest.mark.parametrize("norm", SPARSE)
def test_zero_tiles_skipped_and_results_unchanged(norm):
    """Local attention (each key close to its own query, far from the others):
    the support of every row sits near the diagonal, so most key tiles carry
    no probability at all.  The forward's tile mask must show them, the
    backward that skips them must give what the backward without the mask
    gives (dQ bit for bit: a skipped tile adds exact zeros; dK, dV to fp32
    rounding, their kernel recomputes the scores in another MMA shape), and
    the tail rows must match the oracle."""
    b, h, s, d = 1, 2, 2048, 128
    gen = torch.Generator().manual_seed(7)
    base = torch.randn(b, h, s, d, generator=gen)
    # nearby positions get similar vectors (a slowly rotating direction)
    pos = torch.arange(s, dtype=torch.float32)[:, None]
    freq = torch.rand(d, generator=gen) * 0.05
    smooth = torch.cos(pos * freq) * 2.0
    q = (smooth + 0.3 * base).to(torch.bfloat16).cuda()
    k = (smooth + 0.3 * torch.randn(b, h, s, d, generator=gen)).to(torch.bfloat16).cuda()
    v = torch.randn(b, h, s, d, generator=gen).to(torch.bfloat16).cuda()
    do = torch.randn(b, h, s, d, generator=gen).to(torch.bfloat16).cuda()
    nid, scale = N.NORMALIZER_IDS[norm], d ** -0.5
    o, st, mk, wm, sup = ops.attn_fwd(q, k, v, nid, scale, True, -1, False)
    frac = ops.tile_mask_skipped_fraction(mk, h, b, s, s)
    print(f"{norm}: skipped tile fraction {frac:.3f}")
    assert frac > 0.5
    corr = torch.empty((h, b * s), dtype=torch.float32, device="cuda")
    with_mask = [torch.empty_like(x) for x in (q, k, v)]
    without = [torch.empty_like(x) for x in (q, k, v)]
    ops.attn_bwd_into(do, q, k, v, o, st, corr, *with_mask, nid, scale, True, mask=mk)
    ops.attn_bwd_into(do, q, k, v, o, st, corr, *without, nid, scale, True, mask=None)
    torch.cuda.synchronize()
    assert torch.equal(with_mask[0], without[0])
    for a, e in zip(with_mask[1:], without[1:]):
        err = float((a.float() - e.float()).abs().max())
        assert err <= 1e-2 * float(e.float().abs().max()) + 1e-6
    out = (o, *with_mask)
    _tail_check(norm, q, k, v, do, out, 256, torch.bfloat16, f"local/{norm}")


@pytest.mark.parametrize("norm", SPARSE)
@pytest.mark.parametrize("d,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_saved_wmean_matches_oracle_and_two_pass_backward(norm, d, dtype):
    """The forward's wmean (per row sum_j w_j v_j / sum_j w_j, w = 1[p > 0] for
    sparsemax and sqrt(p) for entmax15) against the oracle's probabilities, and
    the backward that takes its row correction from it (c = dO . wmean, one
    sweep over the keys) against the backward that sweeps twice (c = sum_j w_j
    dP_j / sum_j w_j from the recomputed scores).  The two corrections differ
    by the 16-bit rounding of wmean, so the gradients agree to a stated bound,
    not bit for bit."""
    b, hq, hkv, s = 1, 8, 2, 1024
    q, k, v, do = _inputs((b, hq, s, d), (b, hkv, s, d), dtype, seed=11)
    nid, scale = N.NORMALIZER_IDS[norm], d ** -0.5
    o, st, mk, wm, sup = ops.attn_fwd(q, k, v, nid, scale, True, -1, False)
    assert wm.shape == q.shape
    _, p, _ = oracle.attention_forward(_np(q), _np(k), _np(v), norm, scale=scale, causal=True, return_probs=True)
    w = (p > 0).astype(np.float64) if norm == "sparsemax" else np.sqrt(p)
    vv = np.repeat(_np(v), hq // hkv, axis=1)
    ref = np.einsum("bhqk,bhkd->bhqd", w, vv) / w.sum(-1, keepdims=True)
    err = np.abs(wm.double().cpu().numpy() - ref).max()
    assert err <= 1e-2 * np.abs(ref).max() + 1e-3, f"wmean max err {err:.3e}"
    grads = {}
    for label, wmean in (("one sweep", wm), ("two sweeps", None)):
        corr = torch.empty((hq, b * s), dtype=torch.float32, device="cuda")
        g = [torch.empty_like(x) for x in (q, k, v)]
        ops.attn_bwd_into(do, q, k, v, o, st, corr, *g, nid, scale, True, mask=mk, wmean=wmean)
        grads[label] = (corr, *g)
    torch.cuda.synchronize()
    for name, a, e in zip(("corr", "dq", "dk", "dv"), grads["one sweep"], grads["two sweeps"]):
        err = float((a.float() - e.float()).abs().max())
        assert err <= 1e-2 * float(e.float().abs().max()) + 1e-5, f"{name}: max err {err:.3e}"


def _list_and_tile_grads(q, k, v, do, nid, scale, sup, o, st, mk, wm):
    b, hq, s, _ = q.shape
    grads = {}
    for label, support in (("lists", sup), ("lists again", sup), ("tiles", None)):
        corr = torch.empty((hq, b * s), dtype=torch.float32, device="cuda")
        g = [torch.empty_like(x) for x in (q, k, v)]
        ops.attn_bwd_into(do, q, k, v, o, st, corr, *g, nid, scale, True, mask=mk, wmean=wm, support=support)
        grads[label] = (corr, *g)
    torch.cuda.synchronize()
    for name, a, e in zip(("corr", "dq", "dk", "dv"), grads["lists"], grads["lists again"]):
        assert torch.equal(a, e), f"{name}: the list backward is not run-to-run deterministic"
    for name, a, e in zip(("corr", "dq", "dk", "dv"), grads["lists"], grads["tiles"]):
        err = float((a.float() - e.float()).abs().max())
        assert err <= 1e-2 * float(e.float().abs().max()) + 1e-5, f"{name}: max err {err:.3e}"
    return grads["lists"]


def test_support_lists_only_for_sparsemax():
    """entmax15 takes no support lists (its wider supports make the gathers no
    cheaper than the tile kernels): the workspace query answers 0 bytes."""
    q, k, v, _ = _inputs((1, 4, 256, 128), (1, 2, 256, 128), torch.bfloat16, seed=3)
    assert ops.new_dense_support(q, k, N.NORMALIZER_IDS["entmax15"]).numel() == 0
    assert ops.new_dense_support(q, k, N.NORMALIZER_IDS["sparsemax"]).numel() > 0
    assert ops.attn_fwd(q, k, v, N.NORMALIZER_IDS["entmax15"], 128 ** -0.5, True, -1, False)[4].numel() == 0


def test_support_list_attention_sink():
    """An attention sink: every row keeps key 0, so key 0 has more entries than
    a warp of the list dK/dV kernel sorts (1024); the long-key kernel orders
    its rows with a bitmap.  No fallback is needed, and the results match the
    tile-only backward bit-stably and the oracle."""
    d, dtype = 128, torch.bfloat16
    b, hq, hkv, s = 1, 8, 2, 512
    q, k, v, do = _inputs((b, hq, s, d), (b, hkv, s, d), dtype, seed=19)
    u = torch.randn(d, generator=torch.Generator().manual_seed(5)).to(dtype).cuda()
    q = (q + u).to(dtype)
    k[:, :, 0] = (0.5 * u).to(dtype)
    nid, scale = N.NORMALIZER_IDS["sparsemax"], d ** -0.5
    o, st, mk, wm, sup = ops.attn_fwd(q, k, v, nid, scale, True, -1, False)
    assert not ops.support_overflowed(sup)
    got = _list_and_tile_grads(q, k, v, do, nid, scale, sup, o, st, mk, wm)
    flag = int(sup[:4].view(torch.int32).item())
    assert flag == 0, f"expected no fallback, got flag {flag}"
    ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), "sparsemax", scale=scale, causal=True)
    for name, a, e in zip(("dq", "dk", "dv"), got[1:], ref[1:]):
        assert_close(a, e, dtype, f"sink/{name}")


@pytest.mark.parametrize("d,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_support_list_backward_matches_tile_backward(d, dtype):
    """The forward's support lists (every row's keys with p > 0) drive dQ and
    (transposed to the keys) dK/dV kernels that touch only those entries; they
    must agree with the tile kernels that recompute every tile, give the same
    bits on a second run, and match the oracle.  On N(0, 1) scores no list
    overflows; on nearly flat scores the lists overflow and the backward falls
    back to the tile kernels (checked against the oracle by the wide-support
    tests)."""
    norm = "sparsemax"
    b, hq, hkv, s = 1, 8, 2, 1024
    q, k, v, do = _inputs((b, hq, s, d), (b, hkv, s, d), dtype, seed=13)
    nid, scale = N.NORMALIZER_IDS[norm], d ** -0.5
    o, st, mk, wm, sup = ops.attn_fwd(q, k, v, nid, scale, True, -1, False)
    assert sup.numel() > 0 and not ops.support_overflowed(sup)
    got = _list_and_tile_grads(q, k, v, do, nid, scale, sup, o, st, mk, wm)
    assert not ops.support_overflowed(sup)  # neither a row list nor a key segment overflowed
    ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), norm, scale=scale, causal=True)
    for name, a, e in zip(("dq", "dk", "dv"), got[1:], ref[1:]):
        assert_close(a, e, dtype, f"lists/{name}")
    # nearly flat scores (std ~0.01) at 4096 keys: supports of hundreds of keys
    qw, kw, vw, _ = _inputs((1, 2, 4096, d), (1, 1, 4096, d), dtype, seed=17)
    _, _, _, _, wide = ops.attn_fwd(qw * d ** -0.5, kw * d ** -0.5, vw, nid, scale, True, -1, False)
    assert ops.support_overflowed(wide)
