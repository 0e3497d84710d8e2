"""Generate golden vectors from the reference implementation.

Run in a container where the reference package is importable::

    python tests/golden/make_golden.py /path/to/hf-attention-normalizers

It imports the reference's own eager code -- ``vutils.{softmax_1, sparsemax,
entmax15}``, ``backends.scaled_dot_product_attention``, ``paged.paged_attention``
and the per-sequence loop ``_packed_reference`` of
``tests/test_varlen_attention.py`` -- runs it on the seeds and shapes of the
reference's own tests, and stores inputs and outputs (forward and gradients)
as ``tests/golden/*.npz``.  The reference itself is never needed afterwards:
the committed ``.npz`` files pin the numpy oracle (``oracle/``) and, through
it, the CUDA kernels.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(root: str):
    sys.path.insert(0, root)
    import hf_attention_normalizers  # noqa: F401
    from hf_attention_normalizers import backends, paged, vutils

    spec = importlib.util.spec_from_file_location(
        "ref_test_varlen", os.path.join(root, "tests", "test_varlen_attention.py"))
    tv = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tv)
    return backends, paged, vutils, tv


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def normalizer_cases(vutils, out):
    """Row normalizers on rows with ties, wide ranges and masked tails."""
    fns = {"softmax1": vutils.softmax_1, "sparsemax": vutils.sparsemax, "entmax15": vutils.entmax15}
    g = torch.Generator().manual_seed(5)
    rows = []
    rows.append(torch.randn(64, 33, generator=g, dtype=torch.float64))
    rows.append(torch.randn(16, 300, generator=g, dtype=torch.float64) * 4.0)
    rows.append(torch.randn(16, 300, generator=g, dtype=torch.float64) * 0.05)
    ties = torch.zeros(8, 40, dtype=torch.float64)
    ties[:, :5] = 1.0
    ties[1] = 0.0
    ties[2, 7] = 3.0
    rows.append(ties)
    x = torch.cat([r[:, :33] for r in rows[:1]] + [rows[1][:, :33], rows[2][:, :33], ties[:, :33]])
    masked = x.clone()
    masked[:, 20:] = torch.finfo(torch.float64).min
    for dtype_name, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        for label, inp in (("plain", x), ("masked", masked)):
            xin = inp.to(dtype)
            if dtype == torch.float32:
                xin = torch.where(inp == torch.finfo(torch.float64).min,
                                  torch.full_like(xin, torch.finfo(torch.float32).min), xin)
            dy = torch.randn(xin.shape, generator=g, dtype=torch.float64).to(dtype)
            out[f"norm_{label}_{dtype_name}_x"] = _np(xin)
            out[f"norm_{label}_{dtype_name}_dy"] = _np(dy)
            for name, fn in fns.items():
                xi = xin.clone().requires_grad_(True)
                y = fn(xi, dim=-1)
                y.backward(dy)
                out[f"norm_{label}_{dtype_name}_{name}_y"] = _np(y)
                out[f"norm_{label}_{dtype_name}_{name}_dx"] = _np(xi.grad)


def dense_cases(backends, vutils, out):
    """Dense causal attention, reference test shape (tests/test_hopper_attention.py:15-52)."""
    fns = {"softmax1": vutils.softmax_1, "sparsemax": vutils.sparsemax, "entmax15": vutils.entmax15}
    for tag, shape, kv_heads, seed in (("mha", (1, 2, 129, 32), 2, 31), ("gqa", (1, 4, 70, 64), 2, 3)):
        torch.manual_seed(seed)
        q = torch.randn(shape, dtype=torch.float16).double()
        kshape = (shape[0], kv_heads, shape[2], shape[3])
        k = torch.randn(kshape, dtype=torch.float16).double()
        v = torch.randn(kshape, dtype=torch.float16).double()
        do = torch.randn(shape, dtype=torch.float64)
        out[f"dense_{tag}_q"], out[f"dense_{tag}_k"] = _np(q), _np(k)
        out[f"dense_{tag}_v"], out[f"dense_{tag}_do"] = _np(v), _np(do)
        for name, fn in fns.items():
            qi, ki, vi = (t.clone().requires_grad_(True) for t in (q, k, v))
            o = backends.scaled_dot_product_attention(
                qi, ki, vi, softmax_fn=fn, is_causal=True, scale=shape[-1] ** -0.5,
                enable_gqa=kv_heads != shape[1])
            o.backward(do)
            out[f"dense_{tag}_{name}_o"] = _np(o)
            out[f"dense_{tag}_{name}_dq"] = _np(qi.grad)
            out[f"dense_{tag}_{name}_dk"] = _np(ki.grad)
            out[f"dense_{tag}_{name}_dv"] = _np(vi.grad)


def config1_cases(backends, vutils, out):
    """BASELINE config 1 (fp32, B=2 H=8 S=512 D=128, seed 0): sampled rows + full sums."""
    fns = {"softmax1": vutils.softmax_1, "sparsemax": vutils.sparsemax, "entmax15": vutils.entmax15}
    for name, fn in fns.items():
        torch.manual_seed(0)
        q, k, v = (torch.randn(2, 8, 512, 128, requires_grad=True) for _ in range(3))
        o = backends.scaled_dot_product_attention(q, k, v, softmax_fn=fn, is_causal=True,
                                                   scale=1 / math.sqrt(128))
        g = torch.randn_like(o)
        (o * g).sum().backward()
        for label, t in (("o", o), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
            a = _np(t)
            out[f"config1_{name}_{label}_rows"] = a[:, :, ::61, :].astype(np.float32)
            out[f"config1_{name}_{label}_sum"] = np.array(a.astype(np.float64).sum())
            out[f"config1_{name}_{label}_abssum"] = np.array(np.abs(a.astype(np.float64)).sum())


def varlen_cases(tv, out):
    """tests/test_varlen_attention.py:33-82 shape and seed, evaluated in float64."""
    cu_q = torch.tensor([0, 3, 8], dtype=torch.int32)
    cu_k = torch.tensor([0, 7, 12], dtype=torch.int32)
    out["varlen_cu_q"], out["varlen_cu_k"] = _np(cu_q), _np(cu_k)
    for name in ("softmax1", "sparsemax", "entmax15"):
        torch.manual_seed(59)
        q = torch.randn(8, 4, 32, dtype=torch.float16).double().requires_grad_(True)
        k = torch.randn(12, 2, 32, dtype=torch.float16).double().requires_grad_(True)
        v = torch.randn(12, 2, 32, dtype=torch.float16).double().requires_grad_(True)
        o = tv._packed_reference(q, k, v, cu_q, cu_k, name)
        do = torch.randn(o.shape, generator=torch.Generator().manual_seed(60), dtype=torch.float64)
        o.backward(do)
        for label, t in (("q", q), ("k", k), ("v", v), ("do", do), ("o", o)):
            out[f"varlen_{name}_{label}"] = _np(t)
        for label, t in (("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
            out[f"varlen_{name}_{label}"] = _np(t)


def paged_cases(paged, out):
    """tests/test_paged_attention.py:46-85 (seed 11, fp64) and :144-195 (shared page, seed 23)."""
    for tag, seed, shape, pages, table, lens, bs in (
        ("unique", 11, (2, 4, 2, 8), 16, [[2, 0], [1, 3]], [5, 7], 4),
        ("shared", 23, (2, 4, 2, 32), 16, [[2, 0], [2, 3]], [5, 7], 4),
        ("decode", 7, (3, 8, 1, 64), 64, [[9, 1, 4, 12], [0, 2, 3, 5], [7, 6, 8, 10]], [13, 16, 3], 4),
    ):
        block_table = torch.tensor(table)
        seq_lens = torch.tensor(lens)
        out[f"paged_{tag}_block_table"] = _np(block_table)
        out[f"paged_{tag}_seq_lens"] = _np(seq_lens)
        out[f"paged_{tag}_block_size"] = np.array(bs)
        for name in ("softmax1", "sparsemax", "entmax15"):
            torch.manual_seed(seed)
            q = torch.randn(shape, dtype=torch.float64, requires_grad=True)
            kc = torch.randn(pages, shape[1] // 2, shape[3], dtype=torch.float64, requires_grad=True)
            vc = torch.randn(pages, shape[1] // 2, shape[3], dtype=torch.float64, requires_grad=True)
            o = paged.paged_attention(q, kc, vc, block_table, seq_lens, block_size=bs, normalizer=name)
            do = torch.randn(o.shape, generator=torch.Generator().manual_seed(seed + 1),
                             dtype=torch.float64)
            o.backward(do)
            for label, t in (("q", q), ("kc", kc), ("vc", vc), ("do", do), ("o", o),
                             ("dq", q.grad), ("dkc", kc.grad), ("dvc", vc.grad)):
                out[f"paged_{tag}_{name}_{label}"] = _np(t)


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HFAN_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    torch.set_num_threads(os.cpu_count() or 1)
    backends, paged, vutils, tv = _load_reference(root)
    groups = {
        "normalizers": lambda o: normalizer_cases(vutils, o),
        "dense": lambda o: dense_cases(backends, vutils, o),
        "config1": lambda o: config1_cases(backends, vutils, o),
        "varlen": lambda o: varlen_cases(tv, o),
        "paged": lambda o: paged_cases(paged, o),
    }
    for name, fn in groups.items():
        out: dict[str, np.ndarray] = {}
        fn(out)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
