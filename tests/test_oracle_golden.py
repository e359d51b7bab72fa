"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures come from running the reference implementation on seeded inputs
(``tests/golden/make_golden.py``); every oracle function that the CUDA parity tests
use as the checker is compared with them here, on CPU.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from oracle import blocks as oblocks
from oracle.quant import dequantize_fp8, e4m3_decode, e4m3_encode, quantize_fp8
from tests.conftest import golden


def _gap_aware_same_sets(ids_a, ids_b, scores, k, tol):
    """Index sets equal, except rows whose k-th/(k+1)-th scores are within ``tol``."""
    n_bad = 0
    flat_a = ids_a.reshape(-1, ids_a.shape[-1])
    flat_b = ids_b.reshape(-1, ids_b.shape[-1])
    flat_s = scores.reshape(-1, scores.shape[-1])
    for a, b, s in zip(flat_a, flat_b, flat_s):
        if set(a.tolist()) == set(b.tolist()):
            continue
        srt = np.sort(s)[::-1]
        if k < s.size and abs(srt[k - 1] - srt[k]) <= tol:
            continue
        n_bad += 1
    return n_bad


def test_page_bounds_match_reference():
    g = golden("page_bounds")
    for key in ("64", "32"):
        mins, maxs = oracle.page_bounds(g[f"k{key}"], int(g[f"page{key}"]))
        assert np.array_equal(mins, g[f"min{key}"])
        assert np.array_equal(maxs, g[f"max{key}"])


@pytest.mark.parametrize("topk", [1, 4, 13, 40])
def test_page_select_matches_reference_decode(topk):
    g = golden("page_select")
    ids, scores = oracle.page_select(g["q"], g["mins"], g["maxs"], int(g["page"]), topk, offset=int(g["offset"]))
    ref_ids, ref_scores = g[f"ids_{topk}"], g[f"scores_{topk}"]
    assert ids.shape == ref_ids.shape
    finite = np.isfinite(ref_scores)
    assert np.array_equal(np.isfinite(scores), finite)
    assert np.allclose(scores[finite], ref_scores[finite], rtol=1e-5, atol=1e-5)
    # reference scores are fp32 sums: accept order flips only inside fp32 rounding
    assert _gap_aware_same_sets(ids, ref_ids, scores, ids.shape[-1], 1e-4) == 0
    if topk == 1:
        assert np.array_equal(ids, ref_ids)  # the forced own page


def test_page_select_matches_reference_fp16_inside_sequence():
    g = golden("page_select")
    ids, scores = oracle.page_select(g["q16"], g["mins16"], g["maxs16"], int(g["page"]), 5,
                                     offset=int(g["offset16"]))
    ref_ids = g["ids16_5"]
    assert _gap_aware_same_sets(ids, ref_ids, scores, 5, 1e-4) == 0
    # pages starting after position 100 are invisible
    assert np.all(np.isneginf(scores[..., 7:]))


def test_topk_tie_rule_against_reference_values():
    """torch.topk breaks ties arbitrarily; the oracle takes the lowest index.  The
    selected VALUES must agree, and the oracle's ids must be the lowest-index ones."""
    g = golden("topk_ties")
    s, k = g["scores"], int(g["k"])
    ids = oracle.topk_lowest_index(s, k)
    vals = np.take_along_axis(s, ids, -1)
    assert np.array_equal(vals, g["vals"])
    for row, sel in zip(s, ids):
        kth = row[sel[-1]]
        better = np.nonzero(row > kth)[0]
        assert set(better) <= set(sel.tolist())
        eq = [i for i in sel.tolist() if row[i] == kth]
        assert eq == sorted(np.nonzero(row == kth)[0].tolist())[: len(eq)]


@pytest.mark.parametrize("label,union", [("union", True), ("nounion", False)])
def test_quest_effective_mask_matches_reference(label, union):
    g = golden("quest_variant")
    q, k = g["q"].astype(np.float64), g["k"].astype(np.float64)
    mask = oracle.quest_effective_mask(q, k, int(g["page"]), int(g["topk"]), offset=0, group=2,
                                       gqa_union_mode=union)
    assert np.array_equal(mask, g[f"mask_{label}"])


@pytest.mark.parametrize("label,union", [("union", True), ("nounion", False)])
def test_quest_forward_matches_reference(label, union):
    g = golden("quest_variant")
    q, k, v = (g[x].astype(np.float64) for x in "qkv")
    page, topk = int(g["page"]), int(g["topk"])
    for chunk in (64, 192):
        outs = []
        for start in range(0, q.shape[2], chunk):
            qc = q[:, :, start:start + chunk]
            kc, vc = k[:, :, : start + chunk], v[:, :, : start + chunk]
            mask = oracle.quest_effective_mask(qc, kc, page, topk, offset=start, group=2, gqa_union_mode=union)
            outs.append(oracle.dense_attention(qc, kc, vc, mask=mask))
        out = np.concatenate(outs, axis=2)
        ref = g[f"out{chunk}_{label}"]
        assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-12


def test_block_sparse_matches_reference():
    g = golden("block_sparse")
    out = oracle.block_sparse_attention(g["q"], g["k"], g["v"], g["ids"], block_size=int(g["bs"]))
    assert np.allclose(out, g["out"], atol=2e-6)
    out2 = oracle.block_sparse_attention(g["q2"], g["k2"], g["v2"], g["ids2"], block_size=int(g["bs2"]))
    assert np.allclose(out2, g["out2"], atol=2e-6)
    ids_all = np.broadcast_to(np.arange(4).reshape(1, 1, 1, -1), (1, 4, 128, 4))
    out3 = oracle.block_sparse_attention(g["q"], g["k"], g["v"], ids_all, block_size=int(g["bs"]))
    assert np.allclose(out3, g["out_all"], atol=2e-6)
    # all blocks selected == unmasked dense attention (tests/test_kernels.py:71-83)
    dense = oracle.dense_attention(g["q"], g["k"], g["v"], causal=False)
    assert np.allclose(out3, dense, atol=1e-10)


def test_indexer_matches_reference():
    g = golden("indexer")
    vals, idx = oracle.indexer_topk(g["q"], g["k"], g["w"], int(g["topk"]))
    assert np.allclose(vals, g["vals"], atol=1e-5)
    assert np.array_equal(idx, g["idx"])
    vals2, idx2 = oracle.indexer_topk(g["q2"], g["k2"], g["w2"], int(g["topk2"]))
    assert np.allclose(vals2, g["vals2"], atol=1e-5)
    s = oracle.indexer_scores(g["q2"], g["k2"], g["w2"])
    assert _gap_aware_same_sets(idx2, g["idx2"], s, 10, 1e-5) == 0


def test_dense_matches_reference():
    g = golden("dense")
    assert np.allclose(oracle.dense_attention(g["q"], g["k"], g["v"], causal=True), g["out_causal"], atol=1e-12)
    assert np.allclose(oracle.dense_attention(g["q"], g["k"], g["v"], causal=False), g["out_full"], atol=1e-12)


def test_block_selectors_match_reference():
    g = golden("block_selectors")
    q, k = g["q"].astype(np.float64), g["k"].astype(np.float64)
    mi = oblocks.minference_block_select(q, k, int(g["block"]), int(g["topk"]), sink_size=int(g["sink"]))
    # early query blocks have fewer causal candidates than k: torch.topk then picks
    # arbitrary -inf (future) blocks, the oracle the lowest-index ones.  Both are
    # removed by the causal intersection of effective_mask (selection.py:96-99).
    causal = np.tril(np.ones(mi.shape[-2:], dtype=bool))
    assert np.array_equal(mi & causal, g["mask_minference"] & causal)
    mo = oblocks.moba_select(q, k, int(g["block"]), int(g["topk"]))
    assert np.array_equal(mo & causal, g["mask_moba"] & causal)


def test_fp8_codec_matches_reference():
    g = golden("quant")
    x, grp = g["x"], int(g["group"])
    xg = x.reshape(x.shape[0], -1, grp)
    codes, scale = quantize_fp8(xg, reduce_axes=-1)
    assert np.array_equal(codes.reshape(x.shape), g["codes"])
    assert np.allclose(scale[..., 0], g["scales"], rtol=0, atol=0)
    assert np.array_equal(dequantize_fp8(codes, scale).reshape(x.shape), g["xhat"])
    assert np.array_equal(e4m3_encode(e4m3_decode(np.arange(126, dtype=np.uint8))), np.arange(126, dtype=np.uint8))


def test_paged_decode_matches_reference():
    g = golden("paged_decode")
    q, k, v, pages, page = g["q"], g["k"], g["v"], g["pages"], int(g["page"])
    t, d = k.shape
    # one sequence, one head: logical pages == physical pages
    pool_k = k.reshape(t // page, 1, page, d)
    pool_v = v.reshape(t // page, 1, page, d)
    table = np.arange(t // page)[None]
    out = oracle.paged_sparse_decode(q[None, None], pool_k, pool_v, table, np.array([t]), pages[None, None],
                                     np.array([[len(pages)]]), page_size=page)
    assert np.allclose(out[0, 0], g["out"], atol=1e-6)
    if "out_c_tiled" in g:
        assert np.allclose(out[0, 0], g["out_c_tiled"], atol=2e-4)


def test_lse_merge_equals_attention_over_union():
    rng = np.random.default_rng(0)
    d, n = 16, 50
    q = rng.standard_normal(d)
    ks, vs = rng.standard_normal((n, d)), rng.standard_normal((n, d))
    cuts = [0, 7, 7, 31, 50]  # includes an empty split
    parts = [oracle.attention_with_lse(q, ks[a:b], vs[a:b], 1 / math.sqrt(d)) for a, b in zip(cuts, cuts[1:])]
    o, L = oracle.lse_merge(np.stack([p[0] for p in parts]), np.array([p[1] for p in parts]))
    o_ref, L_ref = oracle.attention_with_lse(q, ks, vs, 1 / math.sqrt(d))
    assert np.allclose(o, o_ref, atol=1e-12) and abs(L - L_ref) < 1e-12
