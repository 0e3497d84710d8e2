"""HuggingFace integration: normalizer registry, AttentionInterface adapters,
backend registration and Qwen3 attention surgery
(reference: hf_attention_normalizers/backends.py:20-1478).

Every adapter keeps the reference's ``(module, query, key, value,
attention_mask, **kwargs) -> (attn_output[B,S,Hq,D], weights)`` contract.
Without a mask, all of them run the fused engine (``hfan::attn_fwd``): GQA is
read in-kernel from the ``[B, Hkv, S, D]`` key/value tensors (no
``repeat_kv`` copy) and the output is written directly in ``[B, S, Hq, D]``
order (no transpose copy).  With an explicit mask the scores are materialised
(cuBLAS matmul) and normalised by the engine's row kernels -- the same
semantics as the reference's eager fallback.
"""

from __future__ import annotations

import math
import weakref
from dataclasses import dataclass
from typing import Callable, Optional, Union

import torch
from torch import nn
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

from . import _native as N
from .kernels._fused import check_dropout
from .vutils import entmax15, softmax_1, sparsemax

SoftmaxLike = Callable[[torch.Tensor, int], torch.Tensor]

SOFTMAX_FUNCTIONS: dict[str, Callable[..., torch.Tensor]] = {
    "vanilla": nn.functional.softmax,
    "softmax": nn.functional.softmax,
    "sparsemax": sparsemax,
    "entmax15": entmax15,
    "softmax1": softmax_1,
    "softmax_1": softmax_1,
}

_FUSED_NAMES = {softmax_1: "softmax1", sparsemax: "sparsemax", entmax15: "entmax15"}


def resolve_softmax_fn(softmax_fn: Union[str, Callable[..., torch.Tensor]]) -> Callable[..., torch.Tensor]:
    if callable(softmax_fn):
        return softmax_fn
    try:
        return SOFTMAX_FUNCTIONS[softmax_fn]
    except KeyError as exc:
        valid = ", ".join(sorted(SOFTMAX_FUNCTIONS))
        raise ValueError(f"Invalid softmax function: {softmax_fn}. Valid options: {valid}") from exc


def _fused_name(softmax_fn) -> Optional[str]:
    if isinstance(softmax_fn, str):
        softmax_fn = SOFTMAX_FUNCTIONS.get(softmax_fn)
    return _FUSED_NAMES.get(softmax_fn)


def _fused_bshd(query, key, value, normalizer, scale, is_causal, window_left=None,
                dropout_p: float = 0.0, key_lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused attention: q [B,Hq,S,D], k/v [B,Hkv,L,D] -> [B,S,Hq,D] contiguous."""
    from . import ops
    from .kernels._fused import dropout_seed

    if query.shape[1] % key.shape[1] != 0:
        raise ValueError("Query heads must be divisible by key/value heads.")
    actual_scale = query.shape[-1] ** -0.5 if scale is None else float(scale)
    window = -1 if window_left is None else int(window_left)
    o = ops.attn_fwd(query, key, value, N.NORMALIZER_IDS[normalizer], actual_scale, bool(is_causal),
                           window, True, float(dropout_p), dropout_seed(query, dropout_p), key_lengths)[0]
    return o


_MASK_CACHE: dict = {"ref": None, "key": None, "value": None}


def _mask_pattern(mask: Optional[torch.Tensor], lq: int, lk: int, source=None):
    """Recognise the masks the fused kernels express without materialising
    anything (every layer of a model gets the same mask, so the answer is
    cached for the last mask seen):

      ("causal", None)         j <= i for every row
      ("padded", lengths)      j <= i and j < lengths[b]: HF's causal mask of a
                               right-padded batch (int32 lengths [B])
      ("window", w)            i - w < j <= i (sliding window of w keys)

    ``mask`` is HF's [B, 1, Lq, Lk] boolean (True = attend) or additive float
    (0 = attend) mask with Lq == Lk.  Anything else returns None: the caller
    then takes the materialised path.  The check itself is one O(B Lq Lk)
    boolean comparison on the device (the reference introspects the mask
    closures instead, backends.py:208-326).  ``source`` is the object the
    caller got (a BlockMask the boolean mask was evaluated from); the cache
    holds a weak reference to it, never an address."""
    if mask is None or lq != lk or torch.compiler.is_compiling():
        return None
    owner = mask if source is None else source
    key = (getattr(owner, "_version", 0), lq, lk)
    ref = _MASK_CACHE["ref"]
    if ref is not None and ref() is owner and _MASK_CACHE["key"] == key:
        return _MASK_CACHE["value"]
    if callable(mask) and not isinstance(mask, torch.Tensor):
        mask = mask()  # evaluated only on a cache miss
    if (not isinstance(mask, torch.Tensor) or mask.ndim != 4 or mask.shape[1] != 1 or mask.shape[-2] != lq
            or mask.shape[-1] < lk):
        return None
    m = mask[:, 0, :, :lk]
    allowed = m if m.dtype == torch.bool else (m == 0)
    i = torch.arange(lq, device=m.device)[:, None]
    j = torch.arange(lk, device=m.device)[None, :]
    causal = j <= i
    lengths = allowed[:, -1, :].sum(-1)
    result = None
    if torch.equal(allowed, (causal[None] & (j[None] < lengths[:, None, None]))):
        full = bool((lengths == lk).all())
        result = ("causal", None) if full else ("padded", lengths.to(torch.int32))
    else:
        w = int(lengths[0])
        if 0 < w < lk and torch.equal(allowed, (causal & (j > i - w))[None].expand_as(allowed)):
            result = ("window", w)
    try:
        _MASK_CACHE["ref"] = weakref.ref(owner)
        _MASK_CACHE["key"], _MASK_CACHE["value"] = key, result
    except TypeError:  # not weak-referenceable: no caching
        _MASK_CACHE["ref"] = None
    return result


def _fused_masked(query, key, value, normalizer, scaling, mask, dropout_p, sliding_window=None, source=None):
    """Fused attention for a recognised mask (see _mask_pattern), else None."""
    pat = _mask_pattern(mask, query.shape[-2], key.shape[-2], source)
    if pat is None or not query.is_cuda or not _fused_dropout_ok(query, dropout_p):
        return None
    kind, arg = pat
    if kind == "causal":
        return _fused_bshd(query, key, value, normalizer, scaling, True, sliding_window, dropout_p)
    if kind == "window" and sliding_window is None:
        return _fused_bshd(query, key, value, normalizer, scaling, True, arg, dropout_p)
    if kind == "padded" and sliding_window is None:
        return _fused_bshd(query, key, value, normalizer, scaling, True, None, dropout_p, key_lengths=arg)
    return None


def _fused_dropout_ok(query: torch.Tensor, dropout_p: float) -> bool:
    """Fused dropout runs on the 16-bit tensor-core kernels (head_dim 64 / 128)."""
    return dropout_p == 0.0 or (query.dtype in (torch.float16, torch.bfloat16) and query.shape[-1] in (64, 128))


def _repeat_kv(x: torch.Tensor, groups: int) -> torch.Tensor:
    if groups == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, groups, s, d).reshape(b, h * groups, s, d)


def scaled_dot_product_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                 softmax_fn: Callable[..., torch.Tensor],
                                 attn_mask: Optional[torch.Tensor] = None, dropout_p: float = 0.0,
                                 is_causal: bool = False, scale: Optional[float] = None,
                                 enable_gqa: bool = False, training: bool = True) -> torch.Tensor:
    """SDPA with a pluggable normalizer (reference backends.py:44-78).

    The causal mask is top-left aligned (``tril``), as in the reference.  The
    fused kernel serves the unmasked / square-causal case; everything else
    materialises the scores and uses the engine's row kernels.
    """
    name = _fused_name(softmax_fn)
    lq, lk = query.size(-2), key.size(-2)
    groups = query.size(-3) // key.size(-3)
    if (name is not None and attn_mask is None and (dropout_p == 0.0 or not training)
            and query.is_cuda and query.dim() == 4 and (not is_causal or lq == lk)
            and (enable_gqa or groups == 1)):
        return _fused_bshd(query, key, value, name, scale, is_causal).transpose(1, 2)
    if enable_gqa:
        key = key.repeat_interleave(groups, -3)
        value = value.repeat_interleave(groups, -3)
    scale_factor = 1 / math.sqrt(query.size(-1)) if scale is None else scale
    attn_weight = query @ key.transpose(-2, -1) * scale_factor
    if is_causal:
        if attn_mask is not None:
            raise ValueError("is_causal=True and attn_mask cannot be used together.")
        causal_mask = torch.ones(lq, lk, dtype=torch.bool, device=query.device).tril(diagonal=0)
        attn_weight = attn_weight.masked_fill(causal_mask.logical_not(), torch.finfo(attn_weight.dtype).min)
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            attn_weight = attn_weight.masked_fill(attn_mask.logical_not(), torch.finfo(attn_weight.dtype).min)
        else:
            attn_weight = attn_weight + attn_mask
    attn_weight = softmax_fn(attn_weight, dim=-1)
    attn_weight = nn.functional.dropout(attn_weight, p=dropout_p, training=training)
    return attn_weight @ value


def _default_causal(module, query, attention_mask) -> bool:
    return query.shape[2] > 1 and attention_mask is None and getattr(module, "is_causal", True)


def sdpa_attention_forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           attention_mask: Optional[torch.Tensor], softmax_fn: Callable[..., torch.Tensor],
                           dropout: float = 0.0, scaling: Optional[float] = None,
                           is_causal: Optional[bool] = None, **kwargs) -> tuple[torch.Tensor, None]:
    """Reference backends.py:81-123; fused when there is no explicit mask."""
    if attention_mask is not None and attention_mask.ndim == 4:
        attention_mask = attention_mask[:, :, :, : key.shape[-2]]
    if is_causal is None:
        is_causal = _default_causal(module, query, attention_mask)
    if torch.jit.is_tracing() and isinstance(is_causal, torch.Tensor):
        is_causal = is_causal.item()
    name = _fused_name(softmax_fn)
    training = getattr(module, "training", False)
    square = query.shape[2] == key.shape[2]
    drop = dropout if training else 0.0
    if name is not None and attention_mask is not None:
        out = _fused_masked(query, key, value, name, scaling, attention_mask, drop, kwargs.get("sliding_window"))
        if out is not None:
            return out, None
    if (name is not None and attention_mask is None and _fused_dropout_ok(query, drop) and query.is_cuda
            and (not is_causal or square)):
        # (the fused causal mask is bottom-right aligned; it equals this path's
        # top-left tril when the lengths agree)
        return _fused_bshd(query, key, value, name, scaling, is_causal, kwargs.get("sliding_window"), drop), None
    out = scaled_dot_product_attention(query, key, value, softmax_fn=softmax_fn, attn_mask=attention_mask,
                                       dropout_p=dropout, scale=scaling, is_causal=is_causal,
                                       training=training, enable_gqa=key.shape[1] != query.shape[1])
    return out.transpose(1, 2).contiguous(), None


def eager_attention_forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                            attention_mask: Optional[torch.Tensor], softmax_fn: Callable[..., torch.Tensor],
                            scaling: float, dropout: float = 0.0, **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference backends.py:861-884: materialises and returns the weights."""
    groups = getattr(module, "num_key_value_groups", query.shape[1] // key.shape[1])
    key_states = _repeat_kv(key, groups)
    value_states = _repeat_kv(value, groups)
    attn_weights = torch.matmul(query, key_states.transpose(2, 3)) * scaling
    if attention_mask is not None:
        mask = attention_mask[:, :, :, : key_states.shape[-2]]
        if mask.dtype == torch.bool:
            # transformers >= 5 builds boolean masks (True = attend).
            attn_weights = attn_weights.masked_fill(mask.logical_not(), torch.finfo(attn_weights.dtype).min)
        else:
            attn_weights = attn_weights + mask
    elif query.shape[2] > 1 and getattr(module, "is_causal", False) and query.shape[2] == key.shape[2]:
        # The mask interface may skip a pure-causal mask; apply it here.
        causal = torch.ones(query.shape[2], key.shape[2], dtype=torch.bool, device=query.device).tril()
        attn_weights = attn_weights.masked_fill(causal.logical_not(), torch.finfo(attn_weights.dtype).min)
    attn_weights = softmax_fn(attn_weights, dim=-1)
    attn_weights = nn.functional.dropout(attn_weights, p=dropout, training=getattr(module, "training", False))
    attn_output = torch.matmul(attn_weights, value_states)
    return attn_output.transpose(1, 2).contiguous(), attn_weights


def _fused_adapter(normalizer: str, label: str):
    fn = {"softmax1": softmax_1, "sparsemax": sparsemax, "entmax15": entmax15}[normalizer]

    def forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                attention_mask: Optional[torch.Tensor], dropout: float = 0.0,
                scaling: Optional[float] = None, is_causal: Optional[bool] = None, **kwargs):
        kwargs.pop("softmax_fn", None)
        kwargs.pop("softmax_n_param", None)
        sliding_window = kwargs.pop("sliding_window", None)
        for unused in ("block_n", "bisection_steps", "max_block_n"):
            kwargs.pop(unused, None)
        drop = dropout if getattr(module, "training", False) else 0.0
        check_dropout(drop)
        if attention_mask is not None:
            out = _fused_masked(query, key, value, normalizer, scaling, attention_mask, drop, sliding_window)
            if out is not None:
                return out, None
        if attention_mask is not None or not query.is_cuda or not _fused_dropout_ok(query, drop):
            # (dropout on 32-bit inputs or other head sizes: materialised path)
            return sdpa_attention_forward(module, query, key, value, attention_mask, softmax_fn=fn,
                                          dropout=dropout, scaling=scaling, is_causal=is_causal, **kwargs)
        if query.shape[-3] % key.shape[-3] != 0:
            raise ValueError("Query heads must be divisible by key/value heads.")
        if is_causal is None:
            is_causal = query.shape[-2] > 1 and getattr(module, "is_causal", True)
        return _fused_bshd(query, key, value, normalizer, scaling, is_causal, sliding_window, drop), None

    forward.__name__ = label
    return forward


hopper_softmax1_attention_forward = _fused_adapter("softmax1", "hopper_softmax1_attention_forward")
hopper_sparsemax_attention_forward = _fused_adapter("sparsemax", "hopper_sparsemax_attention_forward")
hopper_entmax15_attention_forward = _fused_adapter("entmax15", "hopper_entmax15_attention_forward")
triton_sparsemax_attention_forward = _fused_adapter("sparsemax", "triton_sparsemax_attention_forward")
triton_entmax15_attention_forward = _fused_adapter("entmax15", "triton_entmax15_attention_forward")


def flash_attention_softmax_n_forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor,
                                      value: torch.Tensor, attention_mask: Optional[torch.Tensor],
                                      softmax_n_param: Union[int, float] = 1, dropout: float = 0.0,
                                      scaling: Optional[float] = None, is_causal: Optional[bool] = None,
                                      **kwargs) -> tuple[torch.Tensor, None]:
    """The reference's ``*_flash_attention_2`` softmax-n route (backends.py:126-180).

    The engine's fused softmax1 kernel replaces the third-party
    flash-attention-softmax-n package; only n = 1 exists in the engine.
    """
    if query.size(-3) % key.size(-3) != 0:
        raise ValueError(
            "FlashAttention requires the number of query heads to be divisible by "
            f"the number of key/value heads. Got {query.size(-3)} query heads and "
            f"{key.size(-3)} key/value heads.")
    if softmax_n_param != 1:
        raise NotImplementedError("Only softmax_n_param=1 (softmax1) is implemented by the fused engine.")
    kwargs.pop("softmax_fn", None)
    return hopper_softmax1_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                             scaling=scaling, is_causal=is_causal, **kwargs)


def _dense_mask_from_flex_block_mask(block_mask, query_length: int, key_length: int, batch_size: int,
                                     num_heads: int) -> torch.Tensor:
    """Boolean [B, H, Lq, Lk] mask of a Flex BlockMask (block structure and mask_mod)."""
    block_dense = block_mask.to_dense().to(torch.bool)
    qb, kb = block_dense.shape[-2:]
    qbs = (query_length + qb - 1) // qb
    kbs = (key_length + kb - 1) // kb
    dense = block_dense.repeat_interleave(qbs, dim=-2).repeat_interleave(kbs, dim=-1)
    dense = dense[..., :query_length, :key_length].expand(batch_size, num_heads, query_length, key_length)
    dev = dense.device
    bi = torch.arange(batch_size, device=dev)[:, None, None, None]
    hi = torch.arange(num_heads, device=dev)[None, :, None, None]
    qi = torch.arange(query_length, device=dev)[None, None, :, None]
    ki = torch.arange(key_length, device=dev)[None, None, None, :]
    return dense & block_mask.mask_mod(bi, hi, qi, ki)


def flex_attention_normalizer_forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor,
                                      value: torch.Tensor, attention_mask, softmax_fn: Callable[..., torch.Tensor],
                                      dropout: float = 0.0, scaling: Optional[float] = None,
                                      **kwargs) -> tuple[torch.Tensor, None]:
    """``*_flex_attention`` (reference backends.py:475-568): a causal,
    sliding-window or right-padded BlockMask runs the fused kernel (the
    boolean mask is evaluated once per distinct mask to recognise it); other
    BlockMasks are expanded to a dense mask and materialised; without a mask
    the fused kernel runs."""
    try:
        from torch.nn.attention.flex_attention import BlockMask
    except ImportError:  # pragma: no cover
        BlockMask = ()  # type: ignore[assignment]
    kwargs.pop("softmax_n_param", None)
    if isinstance(attention_mask, BlockMask):
        name = _fused_name(softmax_fn)
        training = getattr(module, "training", False)
        if name is not None:
            block_mask = attention_mask

            def one_head():
                return _dense_mask_from_flex_block_mask(block_mask, query.shape[-2], key.shape[-2],
                                                        query.shape[0], 1)

            out = _fused_masked(query, key, value, name, scaling, one_head, dropout if training else 0.0,
                                kwargs.get("sliding_window"), source=attention_mask)
            if out is not None:
                return out, None
        attention_mask = _dense_mask_from_flex_block_mask(attention_mask, query.shape[-2], key.shape[-2],
                                                          query.shape[0], query.shape[1])
        kwargs.pop("is_causal", None)
        return sdpa_attention_forward(module, query, key, value, attention_mask, softmax_fn=softmax_fn,
                                      dropout=dropout, scaling=scaling, is_causal=False, **kwargs)
    return sdpa_attention_forward(module, query, key, value, attention_mask, softmax_fn=softmax_fn,
                                  dropout=dropout, scaling=scaling,
                                  is_causal=False if attention_mask is not None else kwargs.pop("is_causal", None),
                                  **kwargs)


def paged_normalizer_attention_forward(module: nn.Module, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                       attention_mask: Optional[torch.Tensor] = None, cache=None,
                                       cu_seq_lens_q: Optional[torch.Tensor] = None, cu_seq_lens_k=None,
                                       max_seqlen_q: Optional[int] = None, max_seqlen_k=None,
                                       implementation=None, softmax_fn: Callable[..., torch.Tensor] = softmax_1,
                                       **kwargs) -> tuple[torch.Tensor, None]:
    """HuggingFace ``paged_attention`` interface (reference backends.py:791-858):
    cache update, then one packed varlen launch over the continuous batch."""
    if attention_mask is not None:
        raise NotImplementedError(
            "Custom paged_attention supports continuous-batching cumulative-length masks; "
            "arbitrary attention_mask is not supported.")
    if cache is not None:
        k, v = cache.update(k, v, module.layer_idx, **kwargs)
    if isinstance(cu_seq_lens_k, dict):
        layer_type = "sliding_attention" if getattr(module, "sliding_window", None) else "full_attention"
        cu_seq_lens_k = cu_seq_lens_k[layer_type]
        max_seqlen_k = max_seqlen_k[layer_type]
    if cu_seq_lens_q is None or cu_seq_lens_k is None or max_seqlen_q is None or max_seqlen_k is None:
        raise ValueError("paged_attention requires cu_seq_lens_q/k and max_seqlen_q/k.")
    if q.ndim != 4:
        raise ValueError("paged_attention query must have shape [1, heads, total_q, head_dim].")
    packed_query = q.transpose(1, 2).squeeze(0)
    if k.ndim == 4:
        packed_key, packed_value = k.transpose(1, 2).squeeze(0), v.transpose(1, 2).squeeze(0)
    else:
        packed_key, packed_value = k, v
    name = _fused_name(softmax_fn)
    if name is None:
        raise ValueError("paged_attention supports softmax1, sparsemax, or entmax15.")
    from .varlen import varlen_hopper_attention

    output = varlen_hopper_attention(packed_query, packed_key, packed_value, cu_seq_lens_q.to(torch.int32),
                                     cu_seq_lens_k.to(torch.int32), normalizer=name, max_seqlen_q=max_seqlen_q,
                                     max_seqlen_k=max_seqlen_k, scale=getattr(module, "scaling", None),
                                     is_causal=True)
    return output, None


CUSTOM_ATTENTION_FUNCTIONS: dict[str, Callable[..., tuple[torch.Tensor, Optional[torch.Tensor]]]] = {
    "eager": eager_attention_forward,
    "sdpa": sdpa_attention_forward,
    "flash_attention_2": flash_attention_softmax_n_forward,
    "sparsemax_triton": triton_sparsemax_attention_forward,
    "entmax15_triton": triton_entmax15_attention_forward,
    "softmaxn_eager": eager_attention_forward,
    "softmaxn_sdpa": sdpa_attention_forward,
    "softmaxn_flash_attention_2": flash_attention_softmax_n_forward,
    "flex_attention": flex_attention_normalizer_forward,
    "paged_attention": paged_normalizer_attention_forward,
    "sparsemax_flash_attention_3": hopper_sparsemax_attention_forward,
    "entmax15_flash_attention_3": hopper_entmax15_attention_forward,
    "softmax1_flash_attention_3": hopper_softmax1_attention_forward,
}

HF_ATTENTION_BACKENDS = (
    "eager",
    "sdpa",
    "flash_attention_2",
    "flash_attention_3",
    "flex_attention",
    "paged_attention",
    "paged|eager",
    "paged|sdpa",
    "paged|flash_attention_2",
    "paged|flash_attention_3",
)

_SOFTMAX_N = {"softmax1", "softmax_1", "softmax_n"}
_FUSED_NORMS = {"softmax1", "softmax_1", "sparsemax", "entmax15"}


def _softmax_name(softmax_fn) -> str:
    return softmax_fn if isinstance(softmax_fn, str) else getattr(softmax_fn, "__name__", "callable")


def _make_softmax_attention_forward(base_backend: str, softmax_fn: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                                    fallback_backend: str = "sdpa", mode: str = "strict"):
    """Select the adapter for ``<softmax>_<base_backend>`` (reference backends.py:918-992)."""
    resolved = resolve_softmax_fn(softmax_fn)
    name = _softmax_name(softmax_fn)
    softmax_n = name in _SOFTMAX_N
    if base_backend == "eager":
        attention_forward = eager_attention_forward
    elif base_backend == "sdpa":
        attention_forward = sdpa_attention_forward
    elif base_backend == "flash_attention_2" and softmax_n:
        attention_forward = flash_attention_softmax_n_forward
    elif base_backend == "flash_attention_2" and name == "sparsemax":
        attention_forward = hopper_sparsemax_attention_forward
    elif base_backend == "flash_attention_2" and name == "entmax15":
        attention_forward = hopper_entmax15_attention_forward
    elif base_backend == "flex_attention":
        attention_forward = flex_attention_normalizer_forward
    elif (base_backend == "paged_attention" or base_backend.startswith("paged|")) and name in _FUSED_NORMS:
        attention_forward = paged_normalizer_attention_forward
    elif base_backend == "flash_attention_3" and name == "sparsemax":
        attention_forward = hopper_sparsemax_attention_forward
    elif base_backend == "flash_attention_3" and name == "entmax15":
        attention_forward = hopper_entmax15_attention_forward
    elif base_backend == "flash_attention_3" and softmax_n:
        attention_forward = hopper_softmax1_attention_forward
    elif mode == "fallback":
        attention_forward = CUSTOM_ATTENTION_FUNCTIONS[fallback_backend]
    elif mode == "strict":
        def unsupported_attention_forward(*args, **kwargs):
            raise NotImplementedError(
                f"{name}_{base_backend} is registered for HuggingFace compatibility, "
                "but this backend does not have a custom-softmax kernel yet. "
                f"Use mode='fallback' or choose {name}_eager/{name}_sdpa.")

        return unsupported_attention_forward
    else:
        raise ValueError("mode must be 'strict' or 'fallback'")

    def softmax_attention_forward(module: nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                  attention_mask: Optional[torch.Tensor], **kwargs):
        kwargs.pop("softmax_fn", None)
        return attention_forward(module, query, key, value, attention_mask, softmax_fn=resolved,
                                 softmax_n_param=1, **kwargs)

    return softmax_attention_forward


def _register_attention_backend(name: str, attention_forward) -> None:
    if hasattr(ALL_ATTENTION_FUNCTIONS, "register"):
        ALL_ATTENTION_FUNCTIONS.register(name, attention_forward)
    else:
        ALL_ATTENTION_FUNCTIONS[name] = attention_forward
    try:
        from transformers import AttentionMaskInterface
        from transformers.masking_utils import flex_attention_mask, sdpa_mask

        AttentionMaskInterface.register(name, flex_attention_mask if "flex_attention" in name else sdpa_mask)
    except (ImportError, AttributeError):
        pass


def register_softmax_attention_backends(softmax_fn: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                                        prefix: Optional[str] = None, mode: str = "strict",
                                        fallback_backend: str = "sdpa",
                                        include_unsupported: bool = True) -> tuple[str, ...]:
    """Register ``<softmax>_<backend>`` for every HF backend name (reference backends.py:995-1061)."""
    if mode not in {"strict", "fallback"}:
        raise ValueError("mode must be 'strict' or 'fallback'")
    if fallback_backend not in CUSTOM_ATTENTION_FUNCTIONS:
        valid = ", ".join(sorted(CUSTOM_ATTENTION_FUNCTIONS))
        raise ValueError(f"fallback_backend must be one of: {valid}")
    label = prefix or (softmax_fn if isinstance(softmax_fn, str) else getattr(softmax_fn, "__name__", "custom"))
    support_name = softmax_fn if isinstance(softmax_fn, str) else getattr(softmax_fn, "__name__", "custom")
    registered = []
    for backend in HF_ATTENTION_BACKENDS:
        supported = (
            backend in {"eager", "sdpa", "flex_attention", "paged_attention"}
            or (backend == "flash_attention_3" and support_name in _SOFTMAX_N | {"sparsemax", "entmax15"})
            or (backend == "flash_attention_2" and support_name in _SOFTMAX_N | {"sparsemax", "entmax15"})
            or (backend.startswith("paged|") and support_name in _SOFTMAX_N | {"sparsemax", "entmax15"})
        )
        if not supported and not include_unsupported:
            continue
        name = f"{label}_{backend}"
        forward = _make_softmax_attention_forward(backend, softmax_fn=softmax_fn,
                                                  fallback_backend=fallback_backend, mode=mode)
        _register_attention_backend(name, forward)
        registered.append(name)
    return tuple(registered)


def register_softmax1_attention_backends(mode: str = "strict", fallback_backend: str = "sdpa",
                                         include_unsupported: bool = True) -> tuple[str, ...]:
    return register_softmax_attention_backends(softmax_fn="softmax1", mode=mode, fallback_backend=fallback_backend,
                                               include_unsupported=include_unsupported)


def register_sparsemax_attention_backends(mode: str = "strict", fallback_backend: str = "sdpa",
                                          include_unsupported: bool = True,
                                          include_triton: bool = True) -> tuple[str, ...]:
    registered = list(register_softmax_attention_backends(softmax_fn="sparsemax", mode=mode,
                                                          fallback_backend=fallback_backend,
                                                          include_unsupported=include_unsupported))
    if include_triton:
        _register_attention_backend("sparsemax_triton", triton_sparsemax_attention_forward)
        registered.append("sparsemax_triton")
    return tuple(registered)


def register_entmax15_attention_backends(mode: str = "strict", fallback_backend: str = "sdpa",
                                         include_unsupported: bool = True,
                                         include_triton: bool = True) -> tuple[str, ...]:
    registered = list(register_softmax_attention_backends(softmax_fn="entmax15", mode=mode,
                                                          fallback_backend=fallback_backend,
                                                          include_unsupported=include_unsupported))
    if include_triton:
        _register_attention_backend("entmax15_triton", triton_entmax15_attention_forward)
        registered.append("entmax15_triton")
    return tuple(registered)


def softmax_attention_backend_name(base_backend: str = "sdpa",
                                   softmax_fn: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                                   prefix: Optional[str] = None) -> str:
    label = prefix or (softmax_fn if isinstance(softmax_fn, str) else getattr(softmax_fn, "__name__", "custom"))
    if base_backend == "triton" and label in {"sparsemax", "entmax15"}:
        return f"{label}_triton"
    return f"{label}_{base_backend}"


def _register_for(softmax_fn, mode, fallback_backend) -> None:
    if softmax_fn == "sparsemax":
        register_sparsemax_attention_backends(mode=mode, fallback_backend=fallback_backend)
    elif softmax_fn == "entmax15":
        register_entmax15_attention_backends(mode=mode, fallback_backend=fallback_backend)
    elif softmax_fn in {"softmax1", "softmax_1"}:
        register_softmax1_attention_backends(mode=mode, fallback_backend=fallback_backend)
    else:
        register_softmax_attention_backends(softmax_fn=softmax_fn, mode=mode, fallback_backend=fallback_backend)


def _set_implementation(model: nn.Module, name: str) -> None:
    if hasattr(model, "set_attn_implementation"):
        try:
            model.set_attn_implementation(name)
            return
        except ValueError:
            # transformers >= 5 validates any name containing "flash_attention"
            # against its installed flash-attn packages before consulting the
            # registry; the registered name is still served by
            # ALL_ATTENTION_FUNCTIONS, so set it on the config directly.
            if not hasattr(model, "config"):
                raise
    if hasattr(model, "config"):
        model.config._attn_implementation = name
        for sub in model.modules():
            cfg = getattr(sub, "config", None)
            if cfg is not None and cfg is not model.config and hasattr(cfg, "_attn_implementation"):
                cfg._attn_implementation = name
        return
    raise ValueError("model has neither set_attn_implementation nor config._attn_implementation")


def set_softmax_attention_backend(model: nn.Module, base_backend: str = "sdpa",
                                  softmax_fn: Union[str, Callable[..., torch.Tensor]] = "softmax1",
                                  mode: str = "strict", fallback_backend: str = "sdpa") -> nn.Module:
    """Register the normalizer's backends and switch ``model`` to one (reference backends.py:1140-1168)."""
    _register_for(softmax_fn, mode, fallback_backend)
    _set_implementation(model, softmax_attention_backend_name(base_backend, softmax_fn))
    return model


@dataclass(frozen=True)
class AttentionReplacementPolicy:
    name: str
    matches: Callable[[nn.Module], bool]
    build: Callable[[nn.Module, Union[str, Callable[..., torch.Tensor]], str], nn.Module]


def get_attention_forward(attn_implementation: Optional[str]):
    attn_implementation = attn_implementation or "eager"
    if attn_implementation in CUSTOM_ATTENTION_FUNCTIONS:
        return CUSTOM_ATTENTION_FUNCTIONS[attn_implementation]
    if hasattr(ALL_ATTENTION_FUNCTIONS, "get_interface"):
        return ALL_ATTENTION_FUNCTIONS.get_interface(attn_implementation, eager_attention_forward)
    return ALL_ATTENTION_FUNCTIONS.get(attn_implementation, eager_attention_forward)


def _uses_custom_softmax(softmax_name: str) -> bool:
    return softmax_name not in {"vanilla", "softmax"}


def _is_allowed_custom_softmax_backend(softmax_name: str, attn_implementation: str) -> bool:
    return attn_implementation in CUSTOM_ATTENTION_FUNCTIONS or attn_implementation.startswith(f"{softmax_name}_")


from .qwen3 import (  # noqa: E402  (model surgery needs the registry above)
    ATTENTION_REPLACEMENT_POLICIES,
    Qwen3AttentionExtra,
    Qwen3AttentionExtrea,
    apply_softmax1_attention,
    apply_softmax_attention,
    from_pretrained_with_registered_softmax_attention,
    from_pretrained_with_softmax_attention,
    register_attention_replacement_policy,
    replace_attention_modules,
    replace_qwen3_attention_modules,
    supported_attention_policies,
)
