"""ctypes binding of the C ABI in ``include/hfan.h`` (``_lib/libhfan.so``).

The library is built in-tree by ``hf_attention_normalizers_b200.build``.  There
is no fallback: if the library is missing or a call fails, a RuntimeError
names the cause.
"""

from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.environ.get("HFAN_LIBRARY") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libhfan.so")
_lock = threading.Lock()
_lib = None

SOFTMAX1, SPARSEMAX, ENTMAX15 = 0, 1, 2
FLOAT32, FLOAT16, BFLOAT16 = 0, 1, 2

NORMALIZER_IDS = {"softmax1": SOFTMAX1, "softmax_1": SOFTMAX1, "sparsemax": SPARSEMAX, "entmax15": ENTMAX15}


class HfanTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("stride_batch", ctypes.c_int64),
        ("stride_head", ctypes.c_int64),
        ("stride_token", ctypes.c_int64),
    ]


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("normalizer", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("heads_q", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("len_q", ctypes.c_int32),
        ("len_k", ctypes.c_int32),
        ("total_q", ctypes.c_int32),
        ("total_k", ctypes.c_int32),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_k", ctypes.c_void_p),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("window_left", ctypes.c_int32),
        ("grad_dtype", ctypes.c_int32),
        ("tile_mask", ctypes.c_void_p),
        ("dropout_p", ctypes.c_float),
        ("dropout_seed", ctypes.c_void_p),
        ("key_lengths", ctypes.c_void_p),
        ("wmean", HfanTensor),
        ("support", ctypes.c_void_p),
    ]


class PagedDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("normalizer", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("heads_q", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("len_q", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("max_len_k", ctypes.c_int32),
        ("num_cache_tokens", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("grad_dtype", ctypes.c_int32),
    ]


# Every symbol include/hfan.h declares, with its ctypes signature.
_T = HfanTensor
_P = ctypes.c_void_p
SIGNATURES = {
    "hfan_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnDesc), _T, _T, _T, _T, _P, _P]),
    "hfan_attn_tile_mask_words": (ctypes.c_int64, [ctypes.POINTER(AttnDesc)]),
    "hfan_attn_support_bytes": (ctypes.c_int64, [ctypes.POINTER(AttnDesc)]),
    "hfan_attn_bwd": (ctypes.c_int, [ctypes.POINTER(AttnDesc), _T, _T, _T, _T, _T, _P, _P, _T, _T, _T, _P]),
    "hfan_paged_fwd": (ctypes.c_int, [ctypes.POINTER(PagedDesc), _T, _T, _T, _T, _P, _P]),
    "hfan_paged_bwd": (ctypes.c_int, [ctypes.POINTER(PagedDesc), _T, _T, _T, _T, _T, _P, _P, _T, _T, _T, _P]),
    "hfan_paged_decode_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(PagedDesc)]),
    "hfan_paged_decode": (ctypes.c_int, [ctypes.POINTER(PagedDesc), _T, _T, _T, _T, _P, _P, ctypes.c_int64, _P]),
    "hfan_paged_decode_static": (ctypes.c_int, [ctypes.POINTER(PagedDesc), _T, _T, _T, _T, _P, _P]),
    "hfan_rownorm_fwd": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                        _P, ctypes.c_int64, _P, ctypes.c_int64, _P]),
    "hfan_rownorm_bwd": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                        _P, ctypes.c_int64, _P, ctypes.c_int64, _P, ctypes.c_int64, _P]),
    "hfan_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int, _P]),
    "hfan_last_error": (ctypes.c_char_p, []),
    "hfan_abi_version": (ctypes.c_int, []),
}

ABI_VERSION = 2


def library_path() -> str:
    return _LIB_PATH


def lib():
    """Load (once) and return the native library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"hfan native library not found at {_LIB_PATH}; build it with "
                    "`python -m hf_attention_normalizers_b200.build`")
            handle = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            if handle.hfan_abi_version() != ABI_VERSION:
                raise RuntimeError("hfan native library ABI version mismatch; rebuild it")
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().hfan_last_error().decode(errors="replace")
        if rc == 1:
            raise ValueError(msg)
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def device_status(stream: int, clear: bool = True) -> int:
    out = ctypes.c_int(0)
    check(lib().hfan_device_status(ctypes.byref(out), int(clear), ctypes.c_void_p(stream)), "hfan_device_status")
    return out.value
