"""CPU oracle for the Gemma-4 attention hot path (TEST INFRASTRUCTURE ONLY).

This package is a numpy restatement of the reference project's own
high-precision CPU path (``src/gemma4_fa4/masks.py``, ``reference.py`` and
``sparse_schedule.py`` of amazingvince/gemma4-fa4-kernels).  It exists to
*check* the CUDA path, never to *be* it:

* only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
  ``bench.py`` may import it;
* the product package (``gemma4_fa4_kernels_b200``) never imports it and
  fails loudly when its CUDA library is missing.

Parity pin: every function here is checked against golden vectors that
``tests/golden/make_golden.py`` produced by importing the reference package
itself (torch float64 autograd), committed under ``tests/golden/``.
"""

from .masks import gemma4_attention_mask
from .attention import (
    attention_bwd,
    attention_fwd,
    attention_fwd_bwd_varlen,
    attention_fwd_varlen,
    attention_flops,
    mask_aware_pairs,
    valid_pair_count,
)
from .schedule import build_local_sparse_schedule, local_sparse_storage_upper_bound

__all__ = [
    "gemma4_attention_mask",
    "attention_fwd",
    "attention_bwd",
    "attention_fwd_varlen",
    "attention_fwd_bwd_varlen",
    "attention_flops",
    "mask_aware_pairs",
    "valid_pair_count",
    "build_local_sparse_schedule",
    "local_sparse_storage_upper_bound",
]
