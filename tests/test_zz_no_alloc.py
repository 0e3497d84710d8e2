"""The allocation-free decode entry point, hfan_paged_decode_static.

It serves callers that may not allocate device memory while they decode
(serving hot paths, embedders that own the allocator): its
scratch is a fixed array inside the library.  This test drives it through the
C ABI and checks it against hfan_paged_decode, which uses a caller-provided
workspace, on two calls in a row (the second call must not be disturbed by
what the first left in the shared scratch).  It lives in its own file,
collected last, and passes alone or after the other tests.
"""

import ctypes

import pytest
import torch

from hf_attention_normalizers_b200 import _native as N
from hf_attention_normalizers_b200 import ops

pytestmark = pytest.mark.gpu


def _decode_case(seed, lens, hkv=2, g=4, d=128, bs=32):
    gen = torch.Generator().manual_seed(seed)
    lens = torch.tensor(lens, dtype=torch.int32)
    pages = [(int(x) + bs - 1) // bs for x in lens]
    perm = torch.randperm(sum(pages), generator=gen).int()
    table = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    off = 0
    for i, n in enumerate(pages):
        table[i, :n] = perm[off:off + n]
        off += n
    kc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda()
    vc = torch.randn(sum(pages) * bs, hkv, d, generator=gen).to(torch.bfloat16).cuda()
    q = torch.randn(len(lens), hkv * g, 1, d, generator=gen).to(torch.bfloat16).cuda()
    return q, kc, vc, table.cuda(), lens.cuda(), bs


def _run(entry, norm, q, kc, vc, table, lens, bs):
    return _run_with_max(entry, norm, q, kc, vc, table, lens, bs, int(lens.max()))


@pytest.mark.parametrize("norm", ["softmax1", "sparsemax", "entmax15"])
def test_static_scratch_decode_matches_workspace_decode_twice(norm):
    for seed, lens in ((1, [40, 1025, 3000, 7]), (2, [4096, 33, 2048, 1, 999])):
        case = _decode_case(seed, lens)
        o_ref, st_ref = _run("workspace", norm, *case)
        o, st = _run("static", norm, *case)
        # Same kernels on the same inputs, no float atomics: bit-identical
        # outputs and both statistics rows (tau / row max, support / sum).
        assert torch.equal(o, o_ref)
        assert torch.equal(st, st_ref)


def test_static_scratch_rejects_requests_beyond_its_size():
    """512 sequences of 32K-key score rows need far more than the 64 MiB built in."""
    q, kc, vc, table, lens, bs = _decode_case(3, [64])
    n = 512
    qe, le = q.expand(n, -1, -1, -1), lens.expand(n)
    te = torch.zeros(n, 32768 // bs, dtype=torch.int32, device=q.device)  # wide enough for 32K keys
    big = ops._paged_desc(qe, kc, te, le, bs, 32768, N.SPARSEMAX, 128 ** -0.5, True)
    assert N.lib().hfan_paged_decode_workspace_bytes(ctypes.byref(big)) > (64 << 20)
    o = torch.empty(n, q.shape[1], 1, q.shape[3], dtype=q.dtype, device=q.device)
    stats = torch.empty(2, q.shape[1], n, dtype=torch.float32, device=q.device)
    rc = N.lib().hfan_paged_decode_static(ctypes.byref(big), ops._t4(qe), ops._t3(kc), ops._t3(vc), ops._t4(o),
                                          ops._ptr(stats), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1
    assert "built-in scratch" in N.lib().hfan_last_error().decode()


@pytest.mark.parametrize("entry", ["workspace", "static"])
def test_decode_clamps_lengths_beyond_max_len_k(entry):
    """A sequence_lengths entry above max_len_k is clamped to it (it would
    otherwise index past the block-table row and the per-row scratch) and
    the device status word reports it (3)."""
    q, kc, vc, table, lens, bs = _decode_case(4, [300, 1500, 64])
    stream = torch.cuda.current_stream().cuda_stream
    N.device_status(stream, clear=True)
    max_len = 1024
    o_cl, st_cl = _run(entry, "entmax15", q, kc, vc, table, lens.clamp(max=max_len), bs)
    assert N.device_status(stream, clear=True) == 0
    o, st = _run_with_max(entry, "entmax15", q, kc, vc, table, lens, bs, max_len)
    assert N.device_status(stream, clear=True) == 3
    assert torch.equal(o, o_cl) and torch.equal(st, st_cl)


def _run_with_max(entry, norm, q, kc, vc, table, lens, bs, max_len):
    o = torch.empty_like(q)
    b, hq, lq, d = q.shape
    stats = torch.empty((2, hq, b * lq), dtype=torch.float32, device=q.device)
    desc = ops._paged_desc(q, kc, table, lens, bs, max_len, N.NORMALIZER_IDS[norm], d ** -0.5, True)
    lib = N.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if entry == "static":
        rc = lib.hfan_paged_decode_static(ctypes.byref(desc), ops._t4(q), ops._t3(kc), ops._t3(vc), ops._t4(o),
                                          ops._ptr(stats), stream)
    else:
        nbytes = lib.hfan_paged_decode_workspace_bytes(ctypes.byref(desc))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        rc = lib.hfan_paged_decode(ctypes.byref(desc), ops._t4(q), ops._t3(kc), ops._t3(vc), ops._t4(o),
                                   ops._ptr(stats), ops._ptr(ws), nbytes, stream)
    N.check(rc, entry)
    torch.cuda.synchronize()
    return o, stats
