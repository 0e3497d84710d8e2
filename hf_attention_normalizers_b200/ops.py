"""torch.library custom ops over the native library, with fake (meta) kernels
for ``torch.compile(fullgraph=True)`` and autograd formulas.

Ops (namespace ``hfan``):
  attn_fwd / attn_bwd       dense [B, H, S, D] attention
  varlen_fwd / varlen_bwd   packed [T, H, D] attention with cu_seqlens
  paged_fwd / paged_bwd     paged KV cache + block_table
  rownorm_fwd / rownorm_bwd row normalizers on a materialised matrix

Every op launches on the current CUDA stream of its inputs' device; CPU
tensors raise (the engine has no CPU path).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _native as N

_DTYPES = {torch.float32: N.FLOAT32, torch.float16: N.FLOAT16, torch.bfloat16: N.BFLOAT16}


def dtype_id(t: Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def _require_cuda(*ts: Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("hfan attention requires CUDA tensors.")


def _inner_contig(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _t4(t: Optional[Tensor]) -> N.HfanTensor:
    """[B, H, S, D] view -> hfan_tensor."""
    if t is None:
        return N.HfanTensor(None, 0, 0, 0)
    return N.HfanTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _t3(t: Optional[Tensor]) -> N.HfanTensor:
    """Packed [T, H, D] (or cache [P, H, D]) view -> hfan_tensor (no batch stride)."""
    if t is None:
        return N.HfanTensor(None, 0, 0, 0)
    return N.HfanTensor(t.data_ptr(), 0, t.stride(1), t.stride(0))


def _stream(t: Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Optional[Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(None if t is None else t.data_ptr())


# ---------------------------------------------------------------------------
# dense
# ---------------------------------------------------------------------------
def _dense_desc(q, k, normalizer, scale, causal, window_left, grad_dtype=None, mask=None,
                dropout_p=0.0, seed=None, key_lengths=None, wmean=None, support=None) -> N.AttnDesc:
    b, hq, lq, d = q.shape
    return N.AttnDesc(
        dtype=dtype_id(q), normalizer=normalizer, batch=b, heads_q=hq, heads_kv=k.shape[1],
        head_dim=d, len_q=lq, len_k=k.shape[2], total_q=b * lq, total_k=k.shape[0] * k.shape[2], cu_seqlens_q=None,
        cu_seqlens_k=None, scale=float(scale), causal=int(bool(causal)),
        window_left=int(window_left), grad_dtype=dtype_id(q) if grad_dtype is None else grad_dtype,
        tile_mask=_mask_ptr(mask), dropout_p=float(dropout_p),
        dropout_seed=None if (seed is None or dropout_p == 0.0) else seed.data_ptr(),
        key_lengths=None if key_lengths is None else key_lengths.data_ptr(),
        wmean=_t4(_wm_or_none(wmean)), support=_support_ptr(support))


def _support_ptr(support: Optional[Tensor]):
    return None if support is None or support.numel() == 0 else support.data_ptr()


def new_support(q: Tensor, desc: N.AttnDesc) -> Tensor:
    """Workspace for the forward's per-row support lists (hfan_attn_support_bytes;
    empty when the request takes none), which let the backward compute dQ
    from the few keys with p > 0 instead of every key tile."""
    nbytes = int(N.lib().hfan_attn_support_bytes(ctypes.byref(desc)))
    return torch.empty((nbytes,), dtype=torch.uint8, device=q.device)


def new_dense_support(q: Tensor, k: Tensor, normalizer: int) -> Tensor:
    """``new_support`` for a dense [B, H, S, D] request without dropout."""
    return new_support(q, _dense_desc(q, k, normalizer, 1.0, True, -1))


def support_overflowed(support: Tensor) -> bool:
    """True when some row's support list overflowed in the last forward that
    wrote ``support`` (its backward then ran the tile kernels).  Synchronises."""
    return support.numel() > 0 and int(support[:4].view(torch.int32).item()) != 0


def _wm_or_none(wmean: Optional[Tensor]) -> Optional[Tensor]:
    return None if wmean is None or wmean.numel() == 0 else wmean


def new_wmean(q: Tensor, normalizer: int) -> Tensor:
    """The sparse forward's saved w-weighted mean of V, [B, Hq, S, D] in q's
    dtype (empty for softmax1, fp32 inputs and head dims the tensor-core
    kernels do not take: those backwards sweep the keys for the correction)."""
    if normalizer == N.SOFTMAX1 or q.dtype not in (torch.bfloat16, torch.float16) or q.shape[-1] not in (64, 128):
        return q.new_empty((0,))
    return torch.empty(q.shape, dtype=q.dtype, device=q.device)


def mask_words(normalizer: int, heads_q: int, batch: int, len_q: int, len_k: int) -> int:
    """int32 words of the key-tile support mask (hfan_attn_tile_mask_words):
    sparse normalizers, rows of at most 131072 keys; 0 otherwise."""
    if normalizer == N.SOFTMAX1 or len_q <= 0 or len_k <= 0:
        return 0
    tiles = -(-len_k // 128)
    if tiles > 1024:
        return 0
    return heads_q * batch * 2 * (-(-len_q // 128)) * ((tiles + 31) // 32)


def _new_mask(device, normalizer, heads_q, batch, len_q, len_k) -> Tensor:
    return torch.empty((mask_words(normalizer, heads_q, batch, len_q, len_k),), dtype=torch.int32, device=device)


def _mask_ptr(mask: Optional[Tensor]):
    return None if mask is None or mask.numel() == 0 else mask.data_ptr()


def _new_out(q: Tensor, out_bshd: bool) -> Tensor:
    b, h, s, d = q.shape
    if out_bshd:
        return torch.empty((b, s, h, d), dtype=q.dtype, device=q.device)
    return torch.empty_like(q, memory_format=torch.contiguous_format)


def _as_bhsd(o: Tensor, out_bshd: bool) -> Tensor:
    return o.transpose(1, 2) if out_bshd else o


@torch.library.custom_op("hfan::attn_fwd", mutates_args=())
def attn_fwd(q: Tensor, k: Tensor, v: Tensor, normalizer: int, scale: float, causal: bool,
             window_left: int, out_bshd: bool, dropout_p: float = 0.0,
             seed: Optional[Tensor] = None, key_lengths: Optional[Tensor] = None
             ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (o, stats, mask, wmean, support): stats float32 [2, Hq, B*S] (see
    hfan.h), the int32 key-tile support mask of the sparse normalizers (empty
    for softmax1), which the backward uses to skip all-zero tiles, the sparse
    normalizers' w-weighted mean of V (``new_wmean``), which gives the backward
    its row correction without a sweep over the keys, and the support-list
    workspace (``new_support``).  ``dropout_p > 0`` drops
    probabilities with the keep bits generated from the device int64 ``seed``.
    ``key_lengths`` (int32 [B]) gives every sequence its own key count with the
    causal mask aligned at the first key: HF's right-padded batch."""
    _require_cuda(q, k, v)
    q, k, v = _inner_contig(q), _inner_contig(k), _inner_contig(v)
    if key_lengths is not None:
        key_lengths = key_lengths.to(device=q.device, dtype=torch.int32).contiguous()
    o = _new_out(q, out_bshd)
    b, hq, lq, _ = q.shape
    stats = torch.empty((2, hq, b * lq), dtype=torch.float32, device=q.device)
    mask = _new_mask(q.device, normalizer, hq, b, lq, k.shape[2])
    wmean = new_wmean(q, normalizer)
    desc = _dense_desc(q, k, normalizer, scale, causal, window_left, mask=mask, dropout_p=dropout_p, seed=seed,
                       key_lengths=key_lengths, wmean=wmean)
    support = new_support(q, desc)
    desc.support = _support_ptr(support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_fwd(ctypes.byref(desc), _t4(q), _t4(k), _t4(v), _t4(_as_bhsd(o, out_bshd)),
                                      _ptr(stats), _stream(q)), "hfan_attn_fwd")
    return o, stats, mask, wmean, support


@attn_fwd.register_fake
def _(q, k, v, normalizer, scale, causal, window_left, out_bshd, dropout_p=0.0, seed=None, key_lengths=None):
    b, hq, lq, d = q.shape
    o = _new_out(q, out_bshd)
    return (o, q.new_empty((2, hq, b * lq), dtype=torch.float32),
            q.new_empty((mask_words(normalizer, hq, b, lq, k.shape[2]),), dtype=torch.int32),
            new_wmean(q, normalizer),
            new_support(q, _dense_desc(q, k, normalizer, scale, causal, window_left, dropout_p=dropout_p)))


@torch.library.custom_op("hfan::attn_bwd", mutates_args=())
def attn_bwd(do: Tensor, q: Tensor, k: Tensor, v: Tensor, o: Tensor, stats: Tensor, mask: Tensor, normalizer: int,
             scale: float, causal: bool, window_left: int, dropout_p: float = 0.0,
             seed: Optional[Tensor] = None, key_lengths: Optional[Tensor] = None,
             wmean: Optional[Tensor] = None, support: Optional[Tensor] = None) -> tuple[Tensor, Tensor, Tensor]:
    _require_cuda(do, q, k, v, o)
    do, q, k, v, o = (_inner_contig(t) for t in (do, q, k, v, o))
    dq = torch.empty_like(q, memory_format=torch.contiguous_format)
    # keys past a sequence's length get no gradient from the kernels: zeros
    new_kv = torch.zeros_like if key_lengths is not None else torch.empty_like
    dk = new_kv(k, memory_format=torch.contiguous_format)
    dv = new_kv(v, memory_format=torch.contiguous_format)
    if key_lengths is not None:
        key_lengths = key_lengths.to(device=q.device, dtype=torch.int32).contiguous()
    b, hq, lq, _ = q.shape
    corr = torch.empty((hq, b * lq), dtype=torch.float32, device=q.device)
    desc = _dense_desc(q, k, normalizer, scale, causal, window_left, mask=mask, dropout_p=dropout_p, seed=seed,
                       key_lengths=key_lengths, wmean=wmean, support=support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_bwd(ctypes.byref(desc), _t4(q), _t4(k), _t4(v), _t4(o), _t4(do),
                                      _ptr(stats), _ptr(corr), _t4(dq), _t4(dk), _t4(dv), _stream(q)),
                "hfan_attn_bwd")
    return dq, dk, dv


@attn_bwd.register_fake
def _(do, q, k, v, o, stats, mask, normalizer, scale, causal, window_left, dropout_p=0.0, seed=None,
      key_lengths=None, wmean=None, support=None):
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            torch.empty_like(k, memory_format=torch.contiguous_format),
            torch.empty_like(v, memory_format=torch.contiguous_format))


def _attn_setup(ctx, inputs, output):
    q, k, v, normalizer, scale, causal, window_left, out_bshd, dropout_p, seed, key_lengths = inputs
    o, stats, mask, wmean, support = output
    ctx.save_for_backward(q, k, v, o, stats, mask, seed, key_lengths, wmean, support)
    ctx.args = (normalizer, scale, causal, window_left, out_bshd, dropout_p)
    ctx.mark_non_differentiable(stats, mask, wmean, support)
    # no zero-filled gradients for the side outputs (the support workspace
    # alone can be a gigabyte)
    ctx.set_materialize_grads(False)


def _attn_backward(ctx, do, dstats, dmask, dwmean, dsupport):
    if do is None:
        return (None,) * 11
    q, k, v, o, stats, mask, seed, key_lengths, wmean, support = ctx.saved_tensors
    normalizer, scale, causal, window_left, out_bshd, dropout_p = ctx.args
    dq, dk, dv = attn_bwd(_as_bhsd(do, out_bshd), q, k, v, _as_bhsd(o, out_bshd), stats, mask, normalizer,
                          scale, causal, window_left, dropout_p, seed, key_lengths, wmean, support)
    return dq, dk, dv, None, None, None, None, None, None, None, None


torch.library.register_autograd("hfan::attn_fwd", _attn_backward, setup_context=_attn_setup)


def attn_fwd_into(q: Tensor, k: Tensor, v: Tensor, o: Tensor, stats: Tensor, normalizer: int, scale: float,
                  causal: bool, window_left: int = -1, mask: Optional[Tensor] = None,
                  wmean: Optional[Tensor] = None, support: Optional[Tensor] = None) -> None:
    """Forward into caller-owned outputs: ``o`` any [B, Hq, S, D] view with unit
    D stride (for example one rank's slice of a head-major gather buffer), ``stats``
    float32 [2, Hq, B * S], optionally the int32 tile mask (``mask_words`` long)
    and the sparse normalizers' ``wmean`` (``new_wmean``) and support-list
    workspace (``new_support``).  No autograd; no allocation."""
    _require_cuda(q, k, v, o, stats)
    desc = _dense_desc(q, k, normalizer, scale, causal, window_left, mask=mask, wmean=wmean, support=support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_fwd(ctypes.byref(desc), _t4(q), _t4(k), _t4(v), _t4(o), _ptr(stats),
                                      _stream(q)), "hfan_attn_fwd")


def attn_bwd_into(do: Tensor, q: Tensor, k: Tensor, v: Tensor, o: Tensor, stats: Tensor, corr: Tensor,
                  dq: Tensor, dk: Tensor, dv: Tensor, normalizer: int, scale: float, causal: bool,
                  window_left: int = -1, mask: Optional[Tensor] = None, wmean: Optional[Tensor] = None,
                  support: Optional[Tensor] = None) -> None:
    """Backward into caller-owned gradient views (unit D stride) and a float32
    [Hq, B * S] row-correction buffer (``mask``: the forward's tile mask, or
    None; ``wmean`` and ``support``: what the forward wrote, or None).  No
    autograd; no allocation."""
    _require_cuda(do, q, k, v, o, dq, dk, dv)
    desc = _dense_desc(q, k, normalizer, scale, causal, window_left, mask=mask, wmean=wmean, support=support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_bwd(ctypes.byref(desc), _t4(q), _t4(k), _t4(v), _t4(o), _t4(do),
                                      _ptr(stats), _ptr(corr), _t4(dq), _t4(dk), _t4(dv), _stream(q)),
                "hfan_attn_bwd")


# ---------------------------------------------------------------------------
# varlen
# ---------------------------------------------------------------------------
def _varlen_desc(q, k, cu_q, cu_k, max_q, max_k, normalizer, scale, causal, mask=None, wmean=None,
                 support=None, sizes_only=False) -> N.AttnDesc:
    """``sizes_only``: a descriptor for the size queries only (fake tensors have
    no data pointers; the queries test the offsets for null and read nothing)."""
    if sizes_only:
        cq = ck = 1
    else:
        cq, ck = cu_q.data_ptr(), cu_k.data_ptr()
    return N.AttnDesc(
        dtype=dtype_id(q), normalizer=normalizer, batch=cu_q.numel() - 1, heads_q=q.shape[1],
        heads_kv=k.shape[1], head_dim=q.shape[2], len_q=int(max_q), len_k=int(max_k),
        total_q=q.shape[0], total_k=k.shape[0], cu_seqlens_q=cq, cu_seqlens_k=ck,
        scale=float(scale), causal=int(bool(causal)), window_left=0, grad_dtype=dtype_id(q),
        tile_mask=_mask_ptr(mask), wmean=_t3(_wm_or_none(wmean)), support=_support_ptr(support))


@torch.library.custom_op("hfan::varlen_fwd", mutates_args=())
def varlen_fwd(q: Tensor, k: Tensor, v: Tensor, cu_q: Tensor, cu_k: Tensor, max_q: int, max_k: int,
               normalizer: int, scale: float, causal: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (o, stats, mask, wmean, support) as ``attn_fwd`` does, over packed rows."""
    _require_cuda(q, k, v, cu_q, cu_k)
    q, k, v = _inner_contig(q), _inner_contig(k), _inner_contig(v)
    cu_q = cu_q.to(torch.int32).contiguous()
    cu_k = cu_k.to(torch.int32).contiguous()
    o = torch.empty_like(q, memory_format=torch.contiguous_format)
    stats = torch.empty((2, q.shape[1], q.shape[0]), dtype=torch.float32, device=q.device)
    mask = _new_mask(q.device, normalizer, q.shape[1], cu_q.numel() - 1, int(max_q), int(max_k))
    wmean = new_wmean(q, normalizer)
    desc = _varlen_desc(q, k, cu_q, cu_k, max_q, max_k, normalizer, scale, causal, mask=mask, wmean=wmean)
    support = new_support(q, desc)
    desc.support = _support_ptr(support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_fwd(ctypes.byref(desc), _t3(q), _t3(k), _t3(v), _t3(o), _ptr(stats),
                                      _stream(q)), "hfan_attn_fwd(varlen)")
    return o, stats, mask, wmean, support


@varlen_fwd.register_fake
def _(q, k, v, cu_q, cu_k, max_q, max_k, normalizer, scale, causal):
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            q.new_empty((2, q.shape[1], q.shape[0]), dtype=torch.float32),
            q.new_empty((mask_words(normalizer, q.shape[1], cu_q.shape[0] - 1, int(max_q), int(max_k)),),
                        dtype=torch.int32),
            new_wmean(q, normalizer),
            new_support(q, _varlen_desc(q, k, cu_q, cu_k, max_q, max_k, normalizer, scale, causal, sizes_only=True)))


@torch.library.custom_op("hfan::varlen_bwd", mutates_args=())
def varlen_bwd(do: Tensor, q: Tensor, k: Tensor, v: Tensor, o: Tensor, stats: Tensor, mask: Tensor, cu_q: Tensor,
               cu_k: Tensor, max_q: int, max_k: int, normalizer: int, scale: float,
               causal: bool, wmean: Optional[Tensor] = None,
               support: Optional[Tensor] = None) -> tuple[Tensor, Tensor, Tensor]:
    _require_cuda(do, q, k, v, o)
    do, q, k, v, o = (_inner_contig(t) for t in (do, q, k, v, o))
    cu_q = cu_q.to(torch.int32).contiguous()
    cu_k = cu_k.to(torch.int32).contiguous()
    dq = torch.zeros_like(q, memory_format=torch.contiguous_format)
    dk = torch.zeros_like(k, memory_format=torch.contiguous_format)
    dv = torch.zeros_like(v, memory_format=torch.contiguous_format)
    corr = torch.empty((q.shape[1], q.shape[0]), dtype=torch.float32, device=q.device)
    desc = _varlen_desc(q, k, cu_q, cu_k, max_q, max_k, normalizer, scale, causal, mask=mask, wmean=wmean,
                        support=support)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_attn_bwd(ctypes.byref(desc), _t3(q), _t3(k), _t3(v), _t3(o), _t3(do),
                                      _ptr(stats), _ptr(corr), _t3(dq), _t3(dk), _t3(dv), _stream(q)),
                "hfan_attn_bwd(varlen)")
    return dq, dk, dv


@varlen_bwd.register_fake
def _(do, q, k, v, o, stats, mask, cu_q, cu_k, max_q, max_k, normalizer, scale, causal, wmean=None, support=None):
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            torch.empty_like(k, memory_format=torch.contiguous_format),
            torch.empty_like(v, memory_format=torch.contiguous_format))


def _varlen_setup(ctx, inputs, output):
    q, k, v, cu_q, cu_k, max_q, max_k, normalizer, scale, causal = inputs
    o, stats, mask, wmean, support = output
    ctx.save_for_backward(q, k, v, o, stats, mask, cu_q, cu_k, wmean, support)
    ctx.args = (max_q, max_k, normalizer, scale, causal)
    ctx.mark_non_differentiable(stats, mask, wmean, support)
    # no zero-filled gradients for the side outputs (the support workspace
    # alone can be a gigabyte)
    ctx.set_materialize_grads(False)


def _varlen_backward(ctx, do, dstats, dmask, dwmean, dsupport):
    if do is None:
        return (None,) * 10
    q, k, v, o, stats, mask, cu_q, cu_k, wmean, support = ctx.saved_tensors
    max_q, max_k, normalizer, scale, causal = ctx.args
    dq, dk, dv = varlen_bwd(do, q, k, v, o, stats, mask, cu_q, cu_k, max_q, max_k, normalizer, scale, causal,
                            wmean, support)
    return dq, dk, dv, None, None, None, None, None, None, None


torch.library.register_autograd("hfan::varlen_fwd", _varlen_backward, setup_context=_varlen_setup)


# ---------------------------------------------------------------------------
# paged
# ---------------------------------------------------------------------------
def _paged_desc(q, kc, block_table, seq_lens, page_size, max_len_k, normalizer, scale, causal) -> N.PagedDesc:
    b, hq, lq, d = q.shape
    return N.PagedDesc(
        dtype=dtype_id(q), normalizer=normalizer, batch=b, heads_q=hq, heads_kv=kc.shape[1], head_dim=d,
        len_q=lq, page_size=int(page_size), max_blocks=block_table.shape[1], max_len_k=int(max_len_k),
        num_cache_tokens=kc.shape[0], block_table=block_table.data_ptr(), seq_lens=seq_lens.data_ptr(),
        scale=float(scale), causal=int(bool(causal)), grad_dtype=N.FLOAT32)


@torch.library.custom_op("hfan::paged_fwd", mutates_args=())
def paged_fwd(q: Tensor, key_cache: Tensor, value_cache: Tensor, block_table: Tensor, seq_lens: Tensor,
              page_size: int, max_len_k: int, normalizer: int, scale: float,
              causal: bool) -> tuple[Tensor, Tensor]:
    _require_cuda(q, key_cache, value_cache, block_table, seq_lens)
    q, kc, vc = _inner_contig(q), _inner_contig(key_cache), _inner_contig(value_cache)
    bt = block_table.to(torch.int32).contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    o = torch.empty_like(q, memory_format=torch.contiguous_format)
    b, hq, lq, _ = q.shape
    stats = torch.empty((2, hq, b * lq), dtype=torch.float32, device=q.device)
    desc = _paged_desc(q, kc, bt, sl, page_size, max_len_k, normalizer, scale, causal)
    with torch.cuda.device(q.device):
        if lq == 1:
            # serving fast path: split-KV decode with a workspace from the caching allocator
            nbytes = N.lib().hfan_paged_decode_workspace_bytes(ctypes.byref(desc))
            if nbytes > 0:
                ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
                rc = N.lib().hfan_paged_decode(ctypes.byref(desc), _t4(q), _t3(kc), _t3(vc), _t4(o), _ptr(stats),
                                               _ptr(ws), nbytes, _stream(q))
                if rc != 2:  # 2 = shape outside the decode kernel's envelope
                    N.check(rc, "hfan_paged_decode")
                    return o, stats
        N.check(N.lib().hfan_paged_fwd(ctypes.byref(desc), _t4(q), _t3(kc), _t3(vc), _t4(o), _ptr(stats),
                                       _stream(q)), "hfan_paged_fwd")
    return o, stats


@paged_fwd.register_fake
def _(q, key_cache, value_cache, block_table, seq_lens, page_size, max_len_k, normalizer, scale, causal):
    b, hq, lq, _ = q.shape
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            q.new_empty((2, hq, b * lq), dtype=torch.float32))


@torch.library.custom_op("hfan::paged_bwd", mutates_args=())
def paged_bwd(do: Tensor, q: Tensor, key_cache: Tensor, value_cache: Tensor, o: Tensor, stats: Tensor,
              block_table: Tensor, seq_lens: Tensor, page_size: int, max_len_k: int, normalizer: int,
              scale: float, causal: bool) -> tuple[Tensor, Tensor, Tensor]:
    _require_cuda(do, q, key_cache, value_cache, o)
    do, q, kc, vc, o = (_inner_contig(t) for t in (do, q, key_cache, value_cache, o))
    bt = block_table.to(torch.int32).contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    dq = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    dkc = torch.zeros(kc.shape, dtype=torch.float32, device=q.device)
    dvc = torch.zeros(vc.shape, dtype=torch.float32, device=q.device)
    b, hq, lq, _ = q.shape
    corr = torch.empty((hq, b * lq), dtype=torch.float32, device=q.device)
    desc = _paged_desc(q, kc, bt, sl, page_size, max_len_k, normalizer, scale, causal)
    with torch.cuda.device(q.device):
        N.check(N.lib().hfan_paged_bwd(ctypes.byref(desc), _t4(q), _t3(kc), _t3(vc), _t4(o), _t4(do),
                                       _ptr(stats), _ptr(corr), _t4(dq), _t3(dkc), _t3(dvc), _stream(q)),
                "hfan_paged_bwd")
    return dq.to(q.dtype), dkc.to(key_cache.dtype), dvc.to(value_cache.dtype)


@paged_bwd.register_fake
def _(do, q, key_cache, value_cache, o, stats, block_table, seq_lens, page_size, max_len_k, normalizer,
      scale, causal):
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            torch.empty_like(key_cache, memory_format=torch.contiguous_format),
            torch.empty_like(value_cache, memory_format=torch.contiguous_format))


def _paged_setup(ctx, inputs, output):
    q, kc, vc, bt, sl, page_size, max_len_k, normalizer, scale, causal = inputs
    o, stats = output
    ctx.save_for_backward(q, kc, vc, o, stats, bt, sl)
    ctx.args = (page_size, max_len_k, normalizer, scale, causal)
    ctx.mark_non_differentiable(stats)
    ctx.set_materialize_grads(False)


def _paged_backward(ctx, do, dstats):
    if do is None:
        return (None,) * 10
    q, kc, vc, o, stats, bt, sl = ctx.saved_tensors
    page_size, max_len_k, normalizer, scale, causal = ctx.args
    dq, dkc, dvc = paged_bwd(do, q, kc, vc, o, stats, bt, sl, page_size, max_len_k, normalizer, scale, causal)
    return dq, dkc, dvc, None, None, None, None, None, None, None


torch.library.register_autograd("hfan::paged_fwd", _paged_backward, setup_context=_paged_setup)


# ---------------------------------------------------------------------------
# row normalizers
# ---------------------------------------------------------------------------
def _rows(x: Tensor):
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) < x2.shape[1]):
        x2 = x2.contiguous()
    return x2


@torch.library.custom_op("hfan::rownorm_fwd", mutates_args=())
def rownorm_fwd(x: Tensor, normalizer: int) -> Tensor:
    _require_cuda(x)
    x2 = _rows(x)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        N.check(N.lib().hfan_rownorm_fwd(normalizer, dtype_id(x), x2.shape[0], x2.shape[1], _ptr(x2),
                                         max(x2.stride(0), x2.shape[1]), _ptr(y), x2.shape[1], _stream(x)),
                "hfan_rownorm_fwd")
    return y


@rownorm_fwd.register_fake
def _(x, normalizer):
    return torch.empty(x.shape, dtype=x.dtype, device=x.device)


@torch.library.custom_op("hfan::rownorm_bwd", mutates_args=())
def rownorm_bwd(y: Tensor, dy: Tensor, normalizer: int) -> Tensor:
    _require_cuda(y, dy)
    y2 = y.reshape(-1, y.shape[-1]).contiguous()
    dy2 = dy.reshape(-1, dy.shape[-1]).contiguous().to(y.dtype)
    dx = torch.empty(y.shape, dtype=y.dtype, device=y.device)
    with torch.cuda.device(y.device):
        N.check(N.lib().hfan_rownorm_bwd(normalizer, dtype_id(y), y2.shape[0], y2.shape[1], _ptr(y2), y2.shape[1],
                                         _ptr(dy2), dy2.shape[1], _ptr(dx), y2.shape[1], _stream(y)),
                "hfan_rownorm_bwd")
    return dx


@rownorm_bwd.register_fake
def _(y, dy, normalizer):
    return torch.empty(y.shape, dtype=y.dtype, device=y.device)


def _rownorm_setup(ctx, inputs, output):
    ctx.save_for_backward(output)
    ctx.normalizer = inputs[1]


def _rownorm_backward(ctx, dy):
    (y,) = ctx.saved_tensors
    return rownorm_bwd(y, dy, ctx.normalizer), None


torch.library.register_autograd("hfan::rownorm_fwd", _rownorm_backward, setup_context=_rownorm_setup)


def row_normalize(x: Tensor, normalizer: str, dim: int = -1) -> Tensor:
    """Apply a normalizer along ``dim`` with the CUDA row kernels."""
    nid = N.NORMALIZER_IDS[normalizer]
    if dim != -1 and dim != x.dim() - 1:
        return rownorm_fwd(x.movedim(dim, -1).contiguous(), nid).movedim(-1, dim)
    return rownorm_fwd(x, nid)


def tile_mask_skipped_fraction(mask: Tensor, heads_q: int, batch: int, len_q: int, len_k: int,
                               causal: bool = True) -> float:
    """Fraction of the (64-row block, 128-key tile) pairs that the causal mask
    leaves visible whose support bit is clear, i.e. the share of tile work the
    backward skips (dense layout, len_q rows bottom-right aligned to len_k keys)."""
    if mask.numel() == 0:
        return 0.0
    qb = 2 * (-(-len_q // 128))
    kt = -(-len_k // 128)
    w = (kt + 31) // 32
    words = mask.view(heads_q, batch, qb, w).to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(32, device=mask.device, dtype=torch.int64)
    bits = ((words.unsqueeze(-1) >> shifts) & 1).reshape(heads_q, batch, qb, w * 32)[..., :kt].bool()
    rb = torch.arange(qb, device=mask.device)
    last_row = torch.clamp(rb * 64 + 63, max=len_q - 1) + (len_k - len_q)
    first_key = torch.arange(kt, device=mask.device) * 128
    vis = (rb * 64 < len_q)[:, None] & (first_key[None, :] < len_k)
    if causal:
        vis = vis & (first_key[None, :] <= last_row[:, None])
    vis = vis.expand(heads_q, batch, qb, kt)
    total = int(vis.sum())
    return 0.0 if total == 0 else float((vis & ~bits).sum()) / total
