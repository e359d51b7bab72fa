"""Parity at the sizes the bench times (``bench.py`` runs the same checks and reports
them as its ``parity`` block): the GPU result against the CPU oracle on samples of
each full-size workload.

* config 2: 2 of the 16 sequences at T = 65536 (bf16, permuted pool);
* config 3: 64 query rows of T = 32768 in runs of 8 (t < 2048, across 2048, t = T - 1);
* config 4: 8 query blocks spread over T = 131072 (the first and the last), every
  (b, head);
* config 5: 2 sequences at T = 2^20, fp8 KV, against the dequantised oracle.

Selections are bit-exact against the oracle's lowest-index top-k on the kernel's own
fp32 scores (config 4: against the float64 pooled scores, a row may differ only at a
reported near tie); outputs within 2e-3 (bf16) / 1e-2 (fp8) of the float64 oracle, the
fp32-domain decode outputs against the bare tolerance.  The reference's harness
semantics are ``tests/test_kernels.py:31-44`` and ``:126-138``."""

from __future__ import annotations

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


def test_fullsize_quest_decode_c2(cuda):
    from linattn_b200 import QuestDecoder

    c = bench.C2
    cache, qs = bench.build_c2(cuda, 1234, 2)
    dec = QuestDecoder(cache, c["Hq"], c["topk"], sink_pages=c["sink_pages"], q_dtype=torch.bfloat16)
    timed = dec.step(qs[0]).clone()
    r = bench.parity_quest_decode(cache, qs[0], c["topk"], c["sink_pages"], n_splits=dec.n_splits, timed_out=timed)
    assert r["ok"], r
    assert r["timed_output_equal"], r
    assert r["max_abs_fp32"] <= bench.TOL_16, r


def test_fullsize_block_sparse_prefill_c4(cuda):
    from linattn_b200.blocks import block_select, block_sparse_prefill

    c = bench.C4
    q, k, v = bench.build_c4(cuda, 44)
    ids, cnt = block_select(q, k, c["block"], c["topk"], sink_blocks=c["sink_blocks"],
                            window_blocks=c["window_blocks"])
    out = block_sparse_prefill(q, k, v, ids, counts=cnt, rows_per_list=c["block"])
    torch.cuda.synchronize()
    r = bench.parity_block_prefill(q, k, v, ids, cnt, out, c["block"], c["topk"], c["sink_blocks"],
                                   c["window_blocks"])
    assert r["ok"], r
    assert r["sets_mismatch_float64"] <= 0.01 * r["rows_checked"], r


def test_fullsize_dsa_c3(cuda):
    from linattn_b200 import indexer_topk
    from linattn_b200.dsa import token_sparse_attention

    c = bench.C3
    q, k, v, q_idx, codes, scales, w = bench.build_c3(cuda, 33)
    _, ids = indexer_topk(q_idx, codes, w, c["topk"], causal=True, k_scale=scales, scale_group=c["scale_group"],
                          index_dtype=torch.int32, sorted=False)
    out = token_sparse_attention(q, k, v, ids.unsqueeze(1), causal=True)
    torch.cuda.synchronize()
    r = bench.parity_dsa(q, k, v, q_idx, codes, scales, w, ids, out, c["topk"], c["scale_group"])
    assert r["ok"], r


def test_fullsize_fp8_decode_c5(cuda):
    from linattn_b200 import QuestDecoder

    c = bench.C5
    cache, qs, _ = bench.build_c5(cuda, 0, 1, 1, batch=2)
    dec = QuestDecoder(cache, c["Hq"], c["topk"], q_dtype=torch.bfloat16)
    timed = dec.step(qs[0]).clone()
    r = bench.parity_quest_decode(cache, qs[0], c["topk"], 0, n_splits=dec.n_splits, timed_out=timed,
                                  tol=bench.TOL_FP8)
    assert r["ok"], r
