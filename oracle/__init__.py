"""CPU oracle for fused normalizer attention.  TEST INFRASTRUCTURE ONLY.

This package is a numpy restatement of the reference's eager math
(``hf_attention_normalizers/vutils`` and the eager attention loops in
``backends.py`` / ``paged.py`` / the reference tests).  It exists to check the
CUDA kernels: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it.  The product package never imports it and
has no CPU fallback.

Parity of the oracle itself is pinned against golden vectors produced by the
reference implementation (``tests/golden/make_golden.py``).
"""

from .normalizers import (  # noqa: F401
    entmax15,
    entmax15_backward,
    softmax1,
    softmax1_backward,
    sparsemax,
    sparsemax_backward,
    normalize,
    normalize_backward,
)
from .attention import (  # noqa: F401
    attention_forward,
    attention_backward,
    varlen_forward,
    varlen_backward,
    paged_forward,
    paged_backward,
)
from . import philox  # noqa: F401
