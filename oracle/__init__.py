"""CPU oracle for the sparse-attention hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (float64 accumulation) and plain C (``oracle/c``),
the reference algorithms of tongxin/linattn that the CUDA library replaces.  Each
function cites the reference file:line it follows (paths inside the reference
project, e.g. ``src/linattn/kernels/triton/quest_pages.py:38-48``).

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs, and only as the checker or the timed
CPU baseline.  The product path (``linattn_b200``) never imports it and has no CPU
fallback: it raises if its CUDA library is missing.

Parity pinning: ``tests/golden/make_golden.py`` imports the reference package (in
the build container only) and records its outputs on seeded inputs as ``.npz``
fixtures; ``tests/test_oracle_golden.py`` checks every function here against them.
"""

from oracle.quest import (  # noqa: F401
    page_bounds,
    page_scores,
    page_select,
    topk_lowest_index,
    gqa_union,
    quest_effective_mask,
)
from oracle.attention import (  # noqa: F401
    dense_attention,
    block_sparse_attention,
    paged_sparse_decode,
    lse_merge,
    attention_with_lse,
)
from oracle.indexer import indexer_scores, indexer_topk  # noqa: F401
from oracle.quant import e4m3_encode, e4m3_decode, quantize_fp8, dequantize_fp8  # noqa: F401
from oracle.blocks import block_reduce, minference_block_select, moba_select, window_block_select  # noqa: F401
