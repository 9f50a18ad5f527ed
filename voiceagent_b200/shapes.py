"""Row-count buckets for the eager (non-graph) paths.

cuBLAS chooses a GEMM kernel per problem shape, and a shape it has not seen costs
about 0.2 ms of host time per call; cuDNN builds a plan per new convolution shape.
Encode batches and prefill steps have a different token count every time, so their
~75-110 GEMMs per call paid that cost on every step. Rounding the row count up to a
coarse bucket makes shapes repeat: at most 16 rows (up to 256) or 12.5 % of the
rows are padding, and the padding rows are never read by attention nor returned.
"""

from __future__ import annotations


def padded_rows(n: int) -> int:
    """Smallest bucket >= n: multiples of 16 up to 256, then multiples of 2**(floor(log2 n) - 3)."""
    if n <= 0:
        return 0
    if n <= 256:
        return -(-n // 16) * 16
    step = 1 << (n.bit_length() - 4)  # 2**(floor(log2 n) - 3)
    return -(-n // step) * step
