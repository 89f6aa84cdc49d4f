"""Test infrastructure only: the CPU oracle that checks the CUDA kernels.

This package is a numpy fp64 restatement of the reference's ground truth for flash_lab's
attention path (flash_lab/reference.py in tfan2437/flash-attention-lab). Nothing in the product
(the flash_lab package, the C-ABI library) imports it. Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference leg use it, and only as the checker or the timed CPU
baseline, never as the thing measured or shipped.

Parity pin: tests/test_oracle.py checks every function here against golden vectors that the real
reference produced (tests/golden/make_golden.py imports flash_lab.reference and writes the
fixtures), at the reference's own tolerance of atol=1e-12 (tests/test_reference.py:202).
"""

from oracle.attention import (  # noqa: F401
    attention,
    attention_rows,
    attention_tiled,
    causal_mask,
    decode,
    gather_cache,
    merge_partials,
)
