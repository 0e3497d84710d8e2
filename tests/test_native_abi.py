"""CPU checks of the C ABI library: it loads, exports every symbol that
include/hfan.h declares, and rejects invalid requests before touching a GPU."""

import ctypes
import os
import re

import pytest

from hf_attention_normalizers_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "hfan.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int64_t|int|const char\*)\s+(hfan_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    declared = _declared_symbols()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(lib, name), name
        assert name in N.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.hfan_abi_version() == N.ABI_VERSION


def _desc(**kw):
    base = dict(dtype=N.BFLOAT16, normalizer=N.SPARSEMAX, batch=1, heads_q=4, heads_kv=2, head_dim=64,
                len_q=8, len_k=8, total_q=8, cu_seqlens_q=None, cu_seqlens_k=None, scale=0.125, causal=1,
                window_left=0, grad_dtype=N.BFLOAT16)
    base.update(kw)
    return N.AttnDesc(**base)


@pytest.mark.parametrize("kw,msg", [
    (dict(normalizer=7), "unknown normalizer"),
    (dict(dtype=9), "unknown dtype"),
    (dict(heads_q=3, heads_kv=2), "divisible"),
    (dict(head_dim=300), "head_dim"),
    (dict(batch=0), "batch"),
])
def test_invalid_attention_requests_are_rejected_on_host(kw, msg):
    lib = N.lib()
    t = N.HfanTensor(None, 0, 0, 0)
    rc = lib.hfan_attn_fwd(ctypes.byref(_desc(**kw)), t, t, t, t, None, None)
    assert rc == 1
    assert msg in lib.hfan_last_error().decode()


def test_paged_block_table_capacity_is_checked_on_host():
    lib = N.lib()
    t = N.HfanTensor(None, 0, 0, 0)
    d = N.PagedDesc(dtype=N.FLOAT16, normalizer=N.SOFTMAX1, batch=2, heads_q=4, heads_kv=2, head_dim=32,
                    len_q=1, page_size=4, max_blocks=2, max_len_k=9, num_cache_tokens=64,
                    block_table=1, seq_lens=1, scale=0.1, causal=1, grad_dtype=N.FLOAT32)
    rc = lib.hfan_paged_fwd(ctypes.byref(d), t, t, t, t, ctypes.c_void_p(1), None)
    assert rc == 1
    assert "enough blocks" in lib.hfan_last_error().decode()


def test_rownorm_rejects_bad_shapes():
    lib = N.lib()
    rc = lib.hfan_rownorm_fwd(N.SPARSEMAX, N.FLOAT32, 4, 10, None, 5, None, 10, None)
    assert rc == 1


@pytest.mark.parametrize("norm,lq,lk,b,hq", [
    (N.SPARSEMAX, 8192, 8192, 4, 32), (N.ENTMAX15, 77, 190, 1, 4), (N.ENTMAX15, 1, 513, 2, 8),
    (N.SOFTMAX1, 512, 512, 1, 4), (N.SPARSEMAX, 16, 131072, 1, 1), (N.SPARSEMAX, 16, 131073, 1, 1),
])
def test_tile_mask_size_agrees_with_python(norm, lq, lk, b, hq):
    from hf_attention_normalizers_b200 import ops

    d = _desc(normalizer=norm, batch=b, heads_q=hq, heads_kv=1, len_q=lq, len_k=lk, total_q=b * lq)
    assert N.lib().hfan_attn_tile_mask_words(ctypes.byref(d)) == ops.mask_words(norm, hq, b, lq, lk)


def test_tile_mask_rejected_where_none_is_taken():
    lib = N.lib()
    t = N.HfanTensor(None, 0, 0, 0)
    rc = lib.hfan_attn_fwd(ctypes.byref(_desc(normalizer=N.SOFTMAX1, tile_mask=1)), t, t, t, t,
                           ctypes.c_void_p(1), None)
    assert rc == 1 and "tile_mask" in lib.hfan_last_error().decode()
