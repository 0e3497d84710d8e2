"""GPU parity of the CUDA kernels against the numpy oracle and the golden
vectors generated from the reference.

Tolerances (the bar of the engine's target):
  * float32 inputs: |kernel - oracle| <= 1e-5 * max(1, max|oracle|) elementwise.
  * bfloat16: max|kernel - oracle| <= 2e-2 * max|oracle|; float16: 1e-2.
  * every 16-bit case also keeps the reference tests' own bar, mean |err| < 1e-3
    (scaled by max|oracle| for gradients larger than one).
  * sparse thresholds: |tau_kernel - tau_oracle| <= 1e-5 (1 + |tau|) in float32,
    so the zero pattern agrees except for entries within ~1e-5 of tau.
The oracle runs in float64 on the same (dtype-rounded) inputs.
"""

import numpy as np
import pytest
import torch

import oracle
from hf_attention_normalizers_b200 import kernels, ops, varlen
import hf_attention_normalizers_b200 as H
from hf_attention_normalizers_b200 import _native as N

pytestmark = pytest.mark.gpu

NORMS = ("softmax1", "sparsemax", "entmax15")
KERNELS = {
    "softmax1": kernels.hopper_softmax1_attention,
    "sparsemax": kernels.hopper_sparsemax_attention,
    "entmax15": kernels.hopper_entmax15_attention,
}
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 1e-2}


def _np(t):
    return t.detach().double().cpu().numpy()


def assert_close(actual, expected, dtype, what=""):
    a = _np(actual) if isinstance(actual, torch.Tensor) else np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (what, a.shape, e.shape)
    assert np.isfinite(a).all(), f"{what}: non-finite values"
    scale = max(1.0, float(np.abs(e).max())) if dtype == torch.float32 else float(np.abs(e).max()) + 1e-12
    err = np.abs(a - e)
    assert err.max() <= TOL[dtype] * scale, f"{what}: max err {err.max():.3e} vs tol {TOL[dtype] * scale:.3e}"
    if dtype != torch.float32:
        assert err.mean() < 1e-3 * max(1.0, scale), f"{what}: mean err {err.mean():.3e}"


def _inputs(shape_q, shape_kv, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(shape_q, generator=g).to(dtype).cuda()
    k = torch.randn(shape_kv, generator=g).to(dtype).cuda()
    v = torch.randn(shape_kv, generator=g).to(dtype).cuda()
    do = torch.randn(shape_q, generator=g).to(dtype).cuda()
    return q, k, v, do


def _run_dense(norm, q, k, v, do, causal=True, window=None):
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = KERNELS[norm](qr, kr, vr, is_causal=causal, window_left=window)
    o.backward(do)
    torch.cuda.synchronize()
    return o, qr.grad, kr.grad, vr.grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("tag", ["mha", "gqa"])
@pytest.mark.parametrize("norm", NORMS)
def test_dense_matches_reference_golden(golden, norm, tag, dtype):
    """Golden vectors from the reference's eager attention (tests/test_hopper_attention.py shapes)."""
    g = golden("dense")
    q, k, v, do = (torch.tensor(g[f"dense_{tag}_{x}"]).to(dtype).cuda() for x in ("q", "k", "v", "do"))
    out = _run_dense(norm, q, k, v, do)
    if dtype == torch.float32:
        for label, a in zip(("o", "dq", "dk", "dv"), out):
            assert_close(a, g[f"dense_{tag}_{norm}_{label}"], dtype, f"{norm}/{tag}/{label}")
    else:
        ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), norm, causal=True)
        for label, a, e in zip(("o", "dq", "dk", "dv"), out, ref):
            assert_close(a, e, dtype, f"{norm}/{tag}/{label}")


DENSE_CASES = [
    # (B, Hq, Hkv, Lq, Lk, D, causal)
    (2, 4, 2, 200, 200, 64, True),
    (1, 8, 2, 300, 300, 128, True),
    (1, 4, 4, 77, 190, 128, True),     # bottom-right causal with Lq < Lk
    (2, 2, 1, 65, 65, 48, False),
    (1, 4, 1, 1, 513, 128, True),      # decode-like single row
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("case", DENSE_CASES)
@pytest.mark.parametrize("norm", NORMS)
def test_dense_random_matches_oracle(norm, case, dtype):
    b, hq, hkv, lq, lk, d, causal = case
    q, k, v, do = _inputs((b, hq, lq, d), (b, hkv, lk, d), dtype, seed=10 * DENSE_CASES.index(case) + NORMS.index(norm))
    out = _run_dense(norm, q, k, v, do, causal=causal)
    ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), norm, causal=causal)
    for label, a, e in zip(("o", "dq", "dk", "dv"), out, ref):
        assert_close(a, e, dtype, f"{norm}/{case}/{label}")


@pytest.mark.parametrize("norm", NORMS)
def test_sliding_window_matches_oracle(norm):
    q, k, v, do = _inputs((1, 4, 150, 64), (1, 2, 150, 64), torch.bfloat16, seed=3)
    out = _run_dense(norm, q, k, v, do, causal=True, window=20)
    ref = oracle.attention_backward(_np(q), _np(k), _np(v), _np(do), norm, causal=True, window_left=20)
    for label, a, e in zip(("o", "dq", "dk", "dv"), out, ref):
        assert_close(a, e, torch.bfloat16, f"{norm}/window/{label}")


@pytest.mark.parametrize("norm", ("sparsemax", "entmax15"))
def test_sparse_threshold_matches_oracle_fp32(norm):
    """The saved tau equals the oracle's sort-based tau (zero-pattern check)."""
    q, k, v, _ = _inputs((1, 2, 96, 64), (1, 2, 96, 64), torch.float32, seed=11)
    o, stats, _, _, _ = ops.attn_fwd(q, k, v, N.NORMALIZER_IDS[norm], 64 ** -0.5, True, -1, False)
    _, p, s = oracle.attention_forward(_np(q), _np(k), _np(v), norm, causal=True, return_probs=True)
    half = 1.0 if norm == "sparsemax" else 0.5
    with np.errstate(all="ignore"):
        z = (s - s.max(-1, keepdims=True)) * half
        if norm == "sparsemax":
            tau_rel, _ = oracle.normalizers.sparsemax_threshold(z)
        else:
            tau_rel, _ = oracle.normalizers.entmax_threshold(z)
    tau_abs = tau_rel[..., 0] + s.max(-1) * half
    tau_k = stats[0].reshape(1, 2, 96).double().cpu().numpy()
    assert np.all(np.abs(tau_k - tau_abs) <= 1e-5 * (1 + np.abs(tau_abs)))
    support = stats[1].reshape(1, 2, 96).cpu().numpy()
    diff = np.abs(support - (p > 0).sum(-1))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.95


@pytest.mark.parametrize("norm", NORMS)
def test_varlen_matches_reference_golden(golden, norm):
    g = golden("varlen")
    cu_q = torch.tensor(g["varlen_cu_q"]).cuda()
    cu_k = torch.tensor(g["varlen_cu_k"]).cuda()
    for dtype in (torch.float32, torch.float16):
        q, k, v = (torch.tensor(g[f"varlen_{norm}_{x}"]).to(dtype).cuda().requires_grad_(True) for x in "qkv")
        do = torch.tensor(g[f"varlen_{norm}_do"]).to(dtype).cuda()
        o = varlen.varlen_hopper_attention(q, k, v, cu_q, cu_k, norm, max_seqlen_q=8, max_seqlen_k=10)
        o.backward(do)
        if dtype == torch.float32:
            refs = [g[f"varlen_{norm}_{x}"] for x in ("o", "dq", "dk", "dv")]
        else:
            refs = oracle.varlen_backward(_np(q), _np(k), _np(v), _np(do), g["varlen_cu_q"], g["varlen_cu_k"], norm)
        for label, a, e in zip(("o", "dq", "dk", "dv"), (o, q.grad, k.grad, v.grad), refs):
            assert_close(a, e, dtype, f"varlen/{norm}/{label}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("norm", NORMS)
def test_varlen_random_gqa_matches_oracle(norm, dtype):
    gen = torch.Generator().manual_seed(5)
    lens_q = torch.randint(1, 200, (5,), generator=gen)
    lens_k = lens_q + torch.randint(0, 40, (5,), generator=gen)
    cu_q = torch.cat([torch.zeros(1, dtype=torch.long), lens_q.cumsum(0)])
    cu_k = torch.cat([torch.zeros(1, dtype=torch.long), lens_k.cumsum(0)])
    tq, tk = int(cu_q[-1]), int(cu_k[-1])
    q = torch.randn(tq, 8, 128, generator=gen).to(dtype).cuda().requires_grad_(True)
    k = torch.randn(tk, 2, 128, generator=gen).to(dtype).cuda().requires_grad_(True)
    v = torch.randn(tk, 2, 128, generator=gen).to(dtype).cuda().requires_grad_(True)
    do = torch.randn(tq, 8, 128, generator=gen).to(dtype).cuda()
    o = varlen.varlen_hopper_attention(q, k, v, cu_q.cuda().int(), cu_k.cuda().int(), norm)
    o.backward(do)
    refs = oracle.varlen_backward(_np(q), _np(k), _np(v), _np(do), cu_q.numpy(), cu_k.numpy(), norm)
    for label, a, e in zip(("o", "dq", "dk", "dv"), (o, q.grad, k.grad, v.grad), refs):
        assert_close(a, e, dtype, f"varlen-rand/{norm}/{label}")


@pytest.mark.parametrize("tag", ["unique", "shared", "decode"])
@pytest.mark.parametrize("norm", NORMS)
def test_paged_matches_reference_golden(golden, norm, tag):
    g = golden("paged")
    pre = f"paged_{tag}_{norm}_"
    bt = torch.tensor(g[f"paged_{tag}_block_table"]).cuda()
    sl = torch.tensor(g[f"paged_{tag}_seq_lens"]).cuda()
    bs = int(g[f"paged_{tag}_block_size"])
    for dtype in (torch.float32, torch.float16):
        q, kc, vc = (torch.tensor(g[pre + x]).to(dtype).cuda().requires_grad_(True) for x in ("q", "kc", "vc"))
        do = torch.tensor(g[pre + "do"]).to(dtype).cuda()
        o = H.paged_attention(q, kc, vc, bt, sl, block_size=bs, normalizer=norm)
        o.backward(do)
        if dtype == torch.float32:
            refs = [g[pre + x] for x in ("o", "dq", "dkc", "dvc")]
        else:
            refs = oracle.paged_backward(_np(q), _np(kc), _np(vc), _np(do), bt.cpu().numpy(), sl.cpu().numpy(), bs, norm)
        for label, a, e in zip(("o", "dq", "dkc", "dvc"), (o, q.grad, kc.grad, vc.grad), refs):
            assert_close(a, e, dtype, f"paged/{tag}/{norm}/{label}")


def test_paged_rejects_out_of_range_block_table():
    q = torch.randn(1, 2, 1, 32, device="cuda")
    kc = torch.randn(16, 1, 32, device="cuda")
    with pytest.raises(ValueError, match="outside the physical cache"):
        H.paged_attention(q, kc, kc, torch.tensor([[0, 9]], device="cuda"), torch.tensor([8], device="cuda"), 4)


@pytest.mark.parametrize("label", ["plain", "masked"])
@pytest.mark.parametrize("norm", NORMS)
def test_row_normalizers_match_reference_golden(golden, norm, label):
    from hf_attention_normalizers_b200 import vutils

    g = golden("normalizers")
    fn = {"softmax1": vutils.softmax_1, "sparsemax": vutils.sparsemax, "entmax15": vutils.entmax15}[norm]
    x = torch.tensor(g[f"norm_{label}_f32_x"]).cuda().requires_grad_(True)
    dy = torch.tensor(g[f"norm_{label}_f32_dy"]).cuda()
    y = fn(x, dim=-1)
    y.backward(dy)
    assert_close(y, g[f"norm_{label}_f32_{norm}_y"], torch.float32, f"rownorm/{norm}/y")
    assert_close(x.grad, g[f"norm_{label}_f32_{norm}_dx"], torch.float32, f"rownorm/{norm}/dx")


@pytest.mark.parametrize("norm", NORMS)
def test_config1_fp32_matches_reference(golden, norm):
    """BASELINE config 1 (fp32, B=2 H=8 S=512 D=128, seed 0) against the reference's own outputs."""
    g = golden("config1")
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 8, 512, 128) for _ in range(3))
    gr = torch.randn(2, 8, 512, 128)
    q, k, v = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = KERNELS[norm](q, k, v, is_causal=True)
    (o * gr.cuda()).sum().backward()
    for label, a in (("o", o), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
        rows = g[f"config1_{norm}_{label}_rows"]
        assert_close(a[:, :, ::61, :], rows, torch.float32, f"config1/{norm}/{label}")
        assert abs(float(a.double().sum()) - float(g[f"config1_{norm}_{label}_sum"])) < 1e-2


@pytest.mark.parametrize("norm", NORMS)
def test_long_key_row_beyond_old_single_block_limit(norm):
    q = torch.randn(1, 1, 2, 64, device="cuda", dtype=torch.float16, requires_grad=True)
    k = torch.randn(1, 1, 8192, 64, device="cuda", dtype=torch.float16, requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    o = KERNELS[norm](q, k, v, is_causal=True)
    o.float().square().mean().backward()
    ref = oracle.attention_forward(_np(q), _np(k), _np(v), norm, causal=True)
    assert_close(o, ref, torch.float16, "long-row")
    assert all(torch.isfinite(t).all() for t in (q.grad, k.grad, v.grad))


TILE_ORDER_CASES = [
    # (Hq, Hkv): whole tensor vs one KV group at a time
    (8, 8),   # K/V and Q/dO 50 MB each: head-major whole, longest-first per head
    (16, 4),  # K/V 25 MB (longest-first both ways, GQA heads adjacent); Q/dO 100 MB:
              # the dK/dV kernel runs head-major whole and longest-first per group
]


@pytest.mark.parametrize("heads", TILE_ORDER_CASES)
@pytest.mark.parametrize("norm", NORMS)
def test_tile_orders_agree(norm, heads):
    """The tensor-core kernels hand tiles out longest-first across heads when
    the operand they re-read is at most 40 MB, else head by head.  A whole
    12288-token tensor and each of its KV groups alone take different orders;
    heads are independent, so both runs agree bit for bit, for every
    normalizer (the sparse threshold is summed in a fixed order around the row
    maximum).  The whole tensor run twice is bit-identical too.  The last query
    tile is also checked against the oracle."""
    hq, hkv = heads
    grp = hq // hkv
    q, k, v, do = _inputs((1, hq, 12288, 128), (1, hkv, 12288, 128), torch.bfloat16, seed=21 + hq)
    whole = _run_dense(norm, q, k, v, do)
    again = _run_dense(norm, q, k, v, do)
    for label, a, b in zip(("o", "dq", "dk", "dv"), whole, again):
        assert torch.equal(a, b), f"{norm}/rerun/{label}"
    del again
    for kh in range(hkv):
        qs, ks = slice(kh * grp, (kh + 1) * grp), slice(kh, kh + 1)
        one = _run_dense(norm, q[:, qs].contiguous(), k[:, ks].contiguous(), v[:, ks].contiguous(),
                         do[:, qs].contiguous())
        for label, a, b in zip(("o", "dq", "dk", "dv"), whole, one):
            a = a[:, qs] if label in ("o", "dq") else a[:, ks]
            assert torch.equal(a, b), f"{norm}/group {kh}/{label}"
    ref = oracle.attention_forward(_np(q[:, :grp, -128:]), _np(k[:, :1]), _np(v[:, :1]), norm, causal=True)
    assert_close(whole[0][:, :grp, -128:], ref, torch.bfloat16, f"{norm}/last tile")


@pytest.mark.parametrize("norm", NORMS)
def test_torch_compile_fullgraph_bf16(norm):
    def attention(q, k, v):
        return KERNELS[norm](q, k, v, is_causal=True)

    compiled = torch.compile(attention, fullgraph=True)
    q = torch.randn(1, 2, 16, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn_like(q, requires_grad=True)
    v = torch.randn_like(q, requires_grad=True)
    out = compiled(q, k, v)
    out.float().square().mean().backward()
    assert torch.isfinite(out).all()
    assert all(torch.isfinite(x.grad).all() for x in (q, k, v))


@pytest.mark.parametrize("norm", NORMS)
def test_hf_qwen3_backend_matches_materialised_path(norm):
    from transformers.models.qwen3 import Qwen3Config, Qwen3ForCausalLM

    config = Qwen3Config(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=64)
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(config).to(device="cuda", dtype=torch.float32).train()
    ids = torch.randint(0, config.vocab_size, (2, 16), device="cuda")
    H.set_softmax_attention_backend(model, base_backend="flash_attention_3", softmax_fn=norm, mode="strict")
    assert model.config._attn_implementation == f"{norm}_flash_attention_3"
    fused = model(ids).logits
    fused.float().square().mean().backward()
    assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())
    H.set_softmax_attention_backend(model, base_backend="eager", softmax_fn=norm, mode="strict")
    assert model.config._attn_implementation == f"{norm}_eager"
    eager = model(ids).logits
    assert_close(fused, _np(eager), torch.float32, f"qwen3/{norm}")


@pytest.mark.parametrize("norm", NORMS)
def test_paged_decode_serving_shape_matches_oracle(norm):
    """Split-KV decode path: bf16, D=128, GQA 4:1, 32-token pages, permuted pages, long rows."""
    gen = torch.Generator().manual_seed(21)
    lens = torch.tensor([1, 31, 33, 1024, 1025, 3000, 5000], dtype=torch.long)
    bs, hkv, g, d = 32, 2, 4, 128
    pages = [(int(x) + bs - 1) // bs for x in lens]
    perm = torch.randperm(sum(pages), generator=gen)
    table = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    off = 0
    for i, n in enumerate(pages):
        table[i, :n] = perm[off:off + n].int()
        off += n
    kc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda()
    vc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda()
    q = torch.randn(len(lens), hkv * g, 1, d, generator=gen).to(torch.bfloat16).cuda()
    o = H.paged_attention(q, kc, vc, table.cuda(), lens.cuda(), block_size=bs, normalizer=norm)
    ref = oracle.paged_forward(_np(q), _np(kc), _np(vc), table.numpy(), lens.numpy(), bs, norm)
    assert_close(o, ref, torch.bfloat16, f"decode/{norm}")
    assert N.device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("shared", [False, True])
@pytest.mark.parametrize("norm", NORMS)
def test_paged_prefill_tensor_core_route_matches_oracle(norm, shared):
    """Paged prefill + backward on the tensor-core route (pages gathered, dense
    kernels with per-sequence key lengths, dK/dV scattered back): bf16, D=128,
    GQA 4:1, 40 query rows against rows of 40-1100 keys (bottom-right causal;
    every query row sees at least one key: the eager oracle and the kernels
    differ only on rows without any), permuted 32-token pages; with `shared`, two sequences share their first
    pages (atomic accumulation of the page gradients)."""
    gen = torch.Generator().manual_seed(33)
    lens = torch.tensor([40, 300, 517, 1100], dtype=torch.long)
    bs, hkv, g, d, lq = 32, 2, 4, 128, 40
    pages = [(int(x) + bs - 1) // bs for x in lens]
    perm = torch.randperm(sum(pages), generator=gen)
    table = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    off = 0
    for i, n in enumerate(pages):
        table[i, :n] = perm[off:off + n].int()
        off += n
    if shared:
        table[2, :4] = table[3, :4]
    kc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    vc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    q = torch.randn(len(lens), hkv * g, lq, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    do = torch.randn(len(lens), hkv * g, lq, d, generator=gen).to(torch.bfloat16).cuda()
    o = H.paged_attention(q, kc, vc, table.cuda(), lens.cuda(), block_size=bs, normalizer=norm)
    o.backward(do)
    refs = oracle.paged_backward(_np(q), _np(kc), _np(vc), _np(do), table.numpy(), lens.numpy(), bs, norm)
    for label, a, e in zip(("o", "dq", "dkc", "dvc"), (o, q.grad, kc.grad, vc.grad), refs):
        assert_close(a, e, torch.bfloat16, f"paged-tc/{norm}/{label}")
    assert N.device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("norm", NORMS)
def test_hf_continuous_batching_paged_attention_interface(norm):
    """HF `paged_attention` interface (continuous batching): the cache update
    hands back the packed keys/values of every sequence and one varlen launch
    serves the batch (a prefill chunk, a decode token and a full prefill)."""
    from hf_attention_normalizers_b200 import backends

    gen = torch.Generator().manual_seed(44)
    lens_q = torch.tensor([5, 1, 64])
    lens_k = torch.tensor([40, 300, 64])
    cu_q = torch.cat([torch.zeros(1, dtype=torch.long), lens_q.cumsum(0)])
    cu_k = torch.cat([torch.zeros(1, dtype=torch.long), lens_k.cumsum(0)])
    tq, tk, hq, hkv, d = int(cu_q[-1]), int(cu_k[-1]), 8, 2, 128
    q = torch.randn(1, hq, tq, d, generator=gen).to(torch.bfloat16).cuda()
    k_all = torch.randn(1, hkv, tk, d, generator=gen).to(torch.bfloat16).cuda()
    v_all = torch.randn(1, hkv, tk, d, generator=gen).to(torch.bfloat16).cuda()

    class Cache:
        def update(self, k, v, layer_idx, **kw):
            return k_all, v_all

    class Module:
        layer_idx = 0
        scaling = d ** -0.5

    fn = {"softmax1": backends.softmax_1, "sparsemax": backends.sparsemax, "entmax15": backends.entmax15}[norm]
    o, _ = backends.paged_normalizer_attention_forward(
        Module(), q, k_all[:, :, :1], v_all[:, :, :1], None, cache=Cache(), cu_seq_lens_q=cu_q.cuda(),
        cu_seq_lens_k=cu_k.cuda(), max_seqlen_q=int(lens_q.max()), max_seqlen_k=int(lens_k.max()), softmax_fn=fn)
    ref = oracle.varlen_forward(_np(q[0].transpose(0, 1)), _np(k_all[0].transpose(0, 1)), _np(v_all[0].transpose(0, 1)),
                                cu_q.numpy(), cu_k.numpy(), norm)
    assert_close(o, ref, torch.bfloat16, f"hf-paged/{norm}")


@pytest.mark.parametrize("norm", NORMS)
def test_varlen_torch_compile_fullgraph_bf16(norm):
    """tests/test_varlen_attention.py:121-143 of the reference."""
    cu_q = torch.tensor([0, 3, 5], device="cuda", dtype=torch.int32)
    cu_k = torch.tensor([0, 4, 9], device="cuda", dtype=torch.int32)

    def attention(query, key, value):
        return varlen.varlen_hopper_attention(query, key, value, cu_q, cu_k, norm, max_seqlen_q=3, max_seqlen_k=5)

    compiled = torch.compile(attention, fullgraph=True)
    q = torch.randn(5, 4, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(9, 2, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    out = compiled(q, k, v)
    out.float().square().mean().backward()
    assert torch.isfinite(out).all()
    assert all(torch.isfinite(x.grad).all() for x in (q, k, v))
    ref = oracle.varlen_forward(_np(q), _np(k), _np(v), cu_q.cpu().numpy(), cu_k.cpu().numpy(), norm)
    assert_close(out, ref, torch.bfloat16, f"compiled varlen/{norm}")


@pytest.mark.parametrize("norm", NORMS)
def test_paged_torch_compile_fullgraph_bf16(norm):
    """tests/test_paged_attention.py:88-113 of the reference (unique pages)."""
    block_table = torch.tensor([[0, 1], [2, 3]], device="cuda")
    lens = torch.tensor([8, 7], device="cuda")

    def attention(query, key_cache, value_cache):
        return H.paged_triton_attention(query, key_cache, value_cache, block_table, lens, block_size=4,
                                        normalizer=norm, max_key_length=8, assume_unique_pages=True)

    compiled = torch.compile(attention, fullgraph=True)
    q = torch.randn(2, 4, 2, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    kc = torch.randn(16, 2, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    vc = torch.randn_like(kc, requires_grad=True)
    out = compiled(q, kc, vc)
    out.float().square().mean().backward()
    assert torch.isfinite(out).all()
    assert all(torch.isfinite(x.grad).all() for x in (q, kc, vc))
    ref = oracle.paged_forward(_np(q), _np(kc), _np(vc), block_table.cpu().numpy(), lens.cpu().numpy(), 4, norm)
    assert_close(out, ref, torch.bfloat16, f"compiled paged/{norm}")
