"""Times BASELINE config 1 through the reference's own eager torch path.

TEST INFRASTRUCTURE: run by hand in the development container, where the
reference checkout is importable (it is not present where the benchmarks
run); the result is recorded in the repository's notes beside the numpy
restatement's timing that bench.py takes on the GPU box's host cores.

Config 1: q, k, v fp32 N(0,1) with torch.manual_seed(0),
B=2, H=8, S=512, D=128, causal, scale 1/sqrt(D); per normalizer the output of
backends.scaled_dot_product_attention (reference backends.py:44-78 with the
vutils normalizers) and the gradients of sum(out * g), g ~ N(0,1).
All host threads; 1 warm-up, median of 5.

    python oracle/time_reference_config1.py /path/to/reference/checkout
"""

import os
import statistics
import sys
import time


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    from hf_attention_normalizers import backends
    from hf_attention_normalizers.vutils import entmax15, softmax_1, sparsemax

    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 8, 512, 128) for _ in range(3))
    g = torch.randn(2, 8, 512, 128)
    flops = 3.5 * 4.0 * 2 * 8 * 128 * 512 * 513 / 2
    for name, fn in (("softmax1", softmax_1), ("sparsemax", sparsemax), ("entmax15", entmax15)):
        times = []
        for rep in range(6):
            qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
            t0 = time.perf_counter()
            out = backends.scaled_dot_product_attention(qq, kk, vv, fn, is_causal=True, scale=128 ** -0.5)
            (out * g).sum().backward()
            if rep:
                times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
        print(f"{name}: {sec * 1e3:.1f} ms fwd+bwd, {flops / sec / 1e9:.2f} GFLOP/s, "
              f"{torch.get_num_threads()} threads")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HFAN_REFERENCE", "."))
