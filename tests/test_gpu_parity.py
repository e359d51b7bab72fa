"""CUDA parity: every operator against the CPU oracle and the reference's golden outputs.

Tolerances (BASELINE): selected index sets bit-exact on identical fp32 scores;
outputs within 2e-3 max-abs for bf16/fp16 inputs (1e-2 for fp8 KV) against the fp32
/ float64 oracle; fp32 inputs within 2e-5.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import golden

pytestmark = pytest.mark.gpu

TOL_16 = 2e-3
TOL_32 = 2e-5


def assert_close_16(out: torch.Tensor, ref: np.ndarray, tol: float = TOL_16):
    """|out - ref| <= tol + half an ulp of out's dtype at |ref|.

    The kernels accumulate in fp32 and round the result once to the caller's dtype,
    as the reference does (``out.to(q.dtype)``, block_sparse.py:75); that final
    rounding alone reaches 2^-8 |x| for bf16 (2^-11 |x| for fp16), so the BASELINE's
    2e-3 applies to the value before it."""
    half_ulp = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}.get(out.dtype, 0.0)
    err = np.abs(_np(out) - ref)
    bound = tol + half_ulp * np.abs(ref)
    assert np.all(err <= bound), f"max err {err.max():.3e}, worst excess {(err - bound).max():.3e}"


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.dtype in (torch.float16, torch.bfloat16) else t.detach().cpu().numpy()


def _dev(a, dtype=torch.float32, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def _same_sets_gap_aware(ids_a, ids_b, scores, tol):
    bad = 0
    for a, b, s in zip(ids_a.reshape(-1, ids_a.shape[-1]), ids_b.reshape(-1, ids_b.shape[-1]),
                       scores.reshape(-1, scores.shape[-1])):
        sa, sb = set(a[a >= 0].tolist()), set(b[b >= 0].tolist())
        if sa == sb:
            continue
        k = len(sa)
        srt = np.sort(s[np.isfinite(s) | (s > 0)])[::-1]
        if k < srt.size and abs(srt[k - 1] - srt[k]) <= tol:
            continue
        bad += 1
    return bad


# ---------------------------------------------------------------------------------
# page bounds
# ---------------------------------------------------------------------------------
def test_page_bounds_golden(cuda):
    from linattn_b200 import page_bounds

    g = golden("page_bounds")
    mins, maxs = page_bounds(_dev(g["k32"]), int(g["page32"]))
    assert np.array_equal(_np(mins), g["min32"]) and np.array_equal(_np(maxs), g["max32"])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("t,page", [(4096, 16), (1000, 64), (37, 8)])
def test_page_bounds_exact(cuda, dtype, t, page):
    from linattn_b200 import page_bounds

    gen = torch.Generator().manual_seed(t + page)
    k = torch.randn(2, 3, t, 128, generator=gen).to(dtype)
    mins, maxs = page_bounds(k.to(cuda), page)
    om, ox = oracle.page_bounds(k.float().numpy(), page)
    assert np.array_equal(_np(mins), om) and np.array_equal(_np(maxs), ox)


def test_page_bounds_strided_input(cuda):
    from linattn_b200 import page_bounds

    k = torch.randn(2, 40, 4, 64, device=cuda).transpose(1, 2)  # (B,H,T,D) view, non-contiguous
    mins, maxs = page_bounds(k, 16)
    om, ox = oracle.page_bounds(k.cpu().numpy(), 16)
    assert np.array_equal(_np(mins), om) and np.array_equal(_np(maxs), ox)


# ---------------------------------------------------------------------------------
# page select
# ---------------------------------------------------------------------------------
@pytest.mark.parametrize("topk", [1, 4, 13, 40])
def test_page_select_golden_decode(cuda, topk):
    from linattn_b200 import page_select

    g = golden("page_select")
    ids, scores = page_select(_dev(g["q"]), _dev(g["mins"]), _dev(g["maxs"]), int(g["page"]), topk,
                              offset=int(g["offset"]))
    ids, scores = ids.cpu().numpy(), scores.cpu().numpy()
    ref_scores = g[f"scores_{topk}"]
    assert ids.shape == g[f"ids_{topk}"].shape and ids.dtype == np.int64
    fin = np.isfinite(ref_scores)
    assert np.array_equal(np.isfinite(scores), fin) and np.array_equal(np.isposinf(scores), np.isposinf(ref_scores))
    assert np.allclose(scores[fin], ref_scores[fin], rtol=1e-5, atol=1e-5)
    # bit-exact selection on identical fp32 scores (the kernel's own)
    assert np.array_equal(ids, oracle.topk_lowest_index(scores.astype(np.float64), ids.shape[-1]))
    # and the same sets as the reference up to fp32 summation-order near-ties
    assert _same_sets_gap_aware(ids, g[f"ids_{topk}"], scores, 1e-4) == 0


def test_page_select_golden_fp16_inside_sequence(cuda):
    from linattn_b200 import page_select

    g = golden("page_select")
    ids, scores = page_select(_dev(g["q16"], torch.float16), _dev(g["mins16"], torch.float16),
                              _dev(g["maxs16"], torch.float16), int(g["page"]), 5, offset=int(g["offset16"]))
    ids, scores = ids.cpu().numpy(), scores.cpu().numpy()
    assert np.array_equal(ids, oracle.topk_lowest_index(scores.astype(np.float64), 5))
    assert _same_sets_gap_aware(ids, g["ids16_5"], scores, 1e-3) == 0
    assert np.all(np.isneginf(scores[..., 7:]))


def test_page_select_ties_lowest_index(cuda):
    """All pages tie (zero keys): the selection must be the lowest visible indices,
    own page first (+inf)."""
    from linattn_b200 import page_select

    q = torch.randn(1, 2, 3, 64, device=cuda)
    mins = torch.zeros(1, 2, 20, 64, device=cuda)
    ids, scores = page_select(q, mins, mins.clone(), 16, 6, offset=150)
    ids = ids.cpu().numpy()
    for t in range(3):
        own = (150 + t) // 16
        assert ids[0, 0, t, 0] == own
        assert ids[0, 0, t, 1:].tolist() == [i for i in range(20) if i != own][:5]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,tq,n_pages,topk", [(32, 8, 1, 256, 32), (8, 2, 5, 300, 17), (4, 4, 2, 1024, 34)])
def test_quest_select_union_vs_oracle(cuda, dtype, hq, hkv, tq, n_pages, topk):
    from linattn_b200 import _lib as L
    from linattn_b200.quest_pages import quest_select

    gen = torch.Generator().manual_seed(hq * n_pages + tq)
    page, d, b = 16, 128, 2
    t = n_pages * page
    k = torch.randn(b, hkv, t, d, generator=gen).to(dtype)
    q = torch.randn(b, hq, tq, d, generator=gen).to(dtype)
    mins, maxs = oracle.page_bounds(k.float().numpy(), page)
    mins_d, maxs_d = _dev(mins, dtype), _dev(maxs, dtype)
    meta = L.Meta(mins_d.data_ptr(), maxs_d.data_ptr(), mins_d.stride(0), mins_d.stride(2), mins_d.stride(1), None,
                  0, 0, L.dtype_code(mins_d), hkv)
    offset = t - tq - 37
    sel = quest_select(q.to(cuda), meta, page_size=page, n_pages=n_pages, topk=topk, offset=offset,
                       sink_pages=1, group=hq // hkv, seq_len=t)
    scores = sel.scores.cpu().numpy().astype(np.float64)
    ids = sel.ids.cpu().numpy()
    assert np.array_equal(ids, oracle.topk_lowest_index(scores, ids.shape[-1]))
    # scores vs the float64 oracle
    _, o_scores = oracle.page_select(q.float().numpy(), mins, maxs, page, topk, offset=offset, sink_pages=1)
    fin = np.isfinite(o_scores)
    assert np.array_equal(np.isfinite(scores), fin)
    assert np.allclose(scores[fin], o_scores[fin], rtol=2e-5, atol=2e-4)
    # union = oracle union of the kernel's own selection
    union = oracle.gqa_union(np.where(np.take_along_axis(scores, ids, -1) > -np.inf, ids, -1), n_pages, hq // hkv)
    cnt = sel.union_count.cpu().numpy()
    uids = sel.union_ids.cpu().numpy()
    for idx in np.ndindex(*cnt.shape):
        got = uids[idx][: cnt[idx]]
        assert np.all(np.diff(got) > 0)
        assert np.array_equal(got, np.nonzero(union[idx])[0])
    # tokens: pages' rows at positions <= offset + t
    tok = sel.union_tokens.cpu().numpy()
    for idx in np.ndindex(*cnt.shape):
        lim = offset + idx[2] + 1
        exp = sum(max(0, min(page, lim - p * page)) for p in uids[idx][: cnt[idx]])
        assert tok[idx] == exp


# ---------------------------------------------------------------------------------
# block-sparse attention (operator)
# ---------------------------------------------------------------------------------
def test_block_sparse_golden(cuda):
    from linattn_b200 import block_sparse_attention

    g = golden("block_sparse")
    out = block_sparse_attention(_dev(g["q"]), _dev(g["k"]), _dev(g["v"]), _dev(g["ids"], torch.int64),
                                 block_size=int(g["bs"]))
    assert out.dtype == torch.float32
    assert np.abs(_np(out) - g["out"]).max() < TOL_32
    out2 = block_sparse_attention(_dev(g["q2"]), _dev(g["k2"]), _dev(g["v2"]), _dev(g["ids2"], torch.int64),
                                  block_size=int(g["bs2"]))
    assert np.abs(_np(out2) - g["out2"]).max() < TOL_32
    ids_all = torch.arange(4, device=cuda).view(1, 1, 1, -1).expand(1, 4, 128, 4)
    out3 = block_sparse_attention(_dev(g["q"]), _dev(g["k"]), _dev(g["v"]), ids_all, block_size=int(g["bs"]))
    assert np.abs(_np(out3) - g["out_all"]).max() < TOL_32


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_block_sparse_half_matches_reference_test_shape(cuda, dtype):
    """tests/test_kernels.py:126-138 of the reference, at the BASELINE tolerance."""
    from linattn_b200 import block_sparse_attention

    torch.manual_seed(0)
    b, h, t, d, bs = 1, 4, 128, 64, 32
    q = torch.randn(b, h, t, d, dtype=dtype)
    k = torch.randn(b, h, t, d, dtype=dtype)
    v = torch.randn(b, h, t, d, dtype=dtype)
    ids = torch.randint(0, t // bs, (b, h, t, 2))
    ids[..., 1] = torch.arange(t) // bs
    out = block_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), ids.to(cuda), block_size=bs)
    ref = oracle.block_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(),
                                        block_size=bs)
    assert out.dtype == dtype
    assert_close_16(out, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("d", [32, 64, 128, 256])
def test_block_sparse_gqa_shapes(cuda, dtype, d):
    from linattn_b200 import block_sparse_attention

    gen = torch.Generator().manual_seed(d)
    b, hq, hkv, tq, tk, bs, n = 2, 8, 2, 3, 333, 16, 7
    q = torch.randn(b, hq, tq, d, generator=gen).to(dtype)
    k = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    v = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    ids = torch.randint(0, (tk + bs - 1) // bs + 2, (b, hkv, tq, n), generator=gen)  # some past T_k
    out = block_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), ids.to(cuda), block_size=bs)
    ref = oracle.block_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(),
                                        block_size=bs)
    if dtype == torch.float32:
        assert np.abs(_np(out) - ref).max() < TOL_32
    else:
        assert_close_16(out, ref)


def test_block_sparse_all_blocks_is_dense(cuda):
    """``tests/test_kernels.py:71-83``: all blocks selected == unmasked dense attention."""
    from linattn_b200 import block_sparse_attention

    torch.manual_seed(0)
    b, h, t, d, bs = 1, 2, 32, 16, 8
    q, k, v = (torch.randn(b, h, t, d) for _ in range(3))
    ids = torch.arange(t // bs).view(1, 1, 1, -1).expand(b, h, t, -1)
    out = block_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), ids.to(cuda), block_size=bs)
    ref = oracle.dense_attention(q.numpy(), k.numpy(), v.numpy(), causal=False)
    assert np.abs(_np(out) - ref).max() < TOL_32


@pytest.mark.parametrize("splits", [1, 2, 5, 16])
def test_split_kv_invariance(cuda, splits):
    from linattn_b200.block_sparse import kv_contiguous, lists_desc, sparse_attention

    gen = torch.Generator().manual_seed(7)
    b, hq, hkv, d, bs, t = 2, 8, 2, 128, 64, 64 * 40
    q = torch.randn(b, hq, 1, d, generator=gen).to(torch.bfloat16).to(cuda)
    k = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16).to(cuda)
    v = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16).to(cuda)
    ids = torch.randperm(40, generator=gen)[:23].view(1, 1, 23).expand(b, hkv, 23).contiguous().to(cuda)
    lse = torch.empty(b, hq, 1, dtype=torch.float32, device=cuda)
    out = sparse_attention(q, kv_contiguous(k, v, bs), lists_desc(ids, hkv), n_splits=splits, lse_out=lse)
    ref = oracle.block_sparse_attention(_np(q), _np(k), _np(v), ids.cpu().numpy(), block_size=bs)
    assert_close_16(out, ref)
    # lse against the float64 oracle
    for bi in range(b):
        for h in range(hq):
            pos = (ids[bi, h // 4].cpu().numpy()[:, None] * bs + np.arange(bs)).reshape(-1)
            _, l_ref = oracle.attention_with_lse(_np(q)[bi, h, 0], _np(k)[bi, h // 4, pos], _np(v)[bi, h // 4, pos],
                                                 1 / math.sqrt(d))
            assert abs(float(lse[bi, h, 0]) - l_ref) < 1e-3


def test_lse_combine_vs_oracle(cuda):
    from linattn_b200 import lse_combine

    gen = torch.Generator().manual_seed(3)
    o = torch.randn(5, 4, 6, 128, generator=gen)
    lse = torch.randn(5, 4, 6, generator=gen) * 3
    lse[2] = -math.inf  # an empty part
    lse[:, 1, 2] = -math.inf  # an all-empty row
    out, l_out = lse_combine(o.to(cuda), lse.to(cuda))
    o_ref, l_ref = oracle.lse_merge(o.numpy(), lse.numpy())
    assert np.abs(_np(out) - o_ref).max() < 1e-5
    fin = np.isfinite(l_ref)
    assert np.allclose(_np(l_out)[fin], l_ref[fin], atol=1e-5)
    assert np.all(np.isneginf(_np(l_out)[~fin]))


# ---------------------------------------------------------------------------------
# plugin: cuda_quest behind AttentionVariant
# ---------------------------------------------------------------------------------
@pytest.mark.parametrize("label,union", [("union", True), ("nounion", False)])
@pytest.mark.parametrize("chunk", [64, 192])
def test_cuda_quest_variant_golden(cuda, label, union, chunk):
    from linattn_b200 import AttnConfig, build

    g = golden("quest_variant")
    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=32, cache_budget=64,
                     topk_blocks=3, topk_tokens=48, compress_ratio=8, obs_window=16, sink_size=2, stride=4,
                     extras={} if union else {"gqa_union": False})
    var = build("cuda_quest", cfg)
    q, k, v = (_dev(g[x]) for x in "qkv")
    out, state = var.forward(q, k, v, chunk=chunk)
    ref = g[f"out{chunk}_{label}"]
    assert np.abs(_np(out) - ref).max() < TOL_32
    assert set(state) >= {"k", "v", "pos", "page_min", "page_max"}
    st = var.stats()
    assert st["reads_per_query"] > 0 and "pages_per_query" in st


def test_cuda_quest_variant_decode_golden(cuda):
    from linattn_b200 import AttnConfig, build

    g = golden("quest_variant")
    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=32, topk_blocks=3,
                     sink_size=2)
    var = build("cuda_quest", cfg)
    q, k, v = (_dev(g[x]) for x in "qkv")
    _, st = var.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
    od, _ = var.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
    assert np.abs(_np(od) - g["out_decode"]).max() < TOL_32
    assert abs(var.stats()["reads_per_query"] - float(g["reads_decode"])) < 1e-6


def test_cuda_quest_full_budget_is_dense(cuda):
    """``tests/test_budgets.py:64-81``: an unrestricted budget reproduces dense attention."""
    from linattn_b200 import AttnConfig, build

    g = golden("quest_variant")
    q, k, v = (_dev(g[x]) for x in "qkv")
    t = q.shape[2]
    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, topk_blocks=t // 16 + 2)
    out, _ = build("cuda_quest", cfg).forward(q, k, v, chunk=t)
    ref = oracle.dense_attention(g["q"], g["k"], g["v"], causal=True)
    assert np.abs(_np(out) - ref).max() < TOL_32


# ---------------------------------------------------------------------------------
# paged decode (the serving path): C1 and C2 shapes
# ---------------------------------------------------------------------------------
def _make_paged(b, hkv, d, page, lens, dtype, gen, needles=0.0, q_dirs=None, perm=True):
    from linattn_b200 import PagedKVCache

    max_pages = max((x + page - 1) // page for x in lens)
    n_phys = b * max_pages
    cache = PagedKVCache(b, hkv, d, page, max_pages, num_phys_pages=n_phys, dtype=dtype, device="cuda")
    k = torch.randn(n_phys, hkv, page, d, generator=gen)
    v = torch.randn(n_phys, hkv, page, d, generator=gen)
    table = torch.randperm(n_phys, generator=gen) if perm else torch.arange(n_phys)
    table = table.view(b, max_pages).to(torch.int32)
    if needles > 0 and q_dirs is not None:
        n_needle = max(1, int(needles * n_phys))
        pick = torch.randperm(n_phys, generator=gen)[:n_needle]
        for p in pick.tolist():
            k[p] += (0.3 * math.sqrt(d)) * q_dirs[:, None, :]
    cache.k_pool.copy_(k.to(dtype))
    cache.v_pool.copy_(v.to(dtype))
    cache.set_page_table(table, lens)
    cache.refresh_meta()
    return cache, table


def _check_decode(cache, table, q, topk, sink, tol, chunks=None):
    from linattn_b200 import QuestDecoder

    hq = q.shape[1]
    dec = QuestDecoder(cache, hq, topk, sink_pages=sink, q_dtype=q.dtype, keep_scores=True, select_chunks=chunks)
    if chunks is not None:
        assert dec.chunks == chunks
    out = dec.step(q)
    torch.cuda.synchronize()
    b, hkv, page, d = cache.batch, cache.n_kv_heads, cache.page_size, cache.head_dim
    lens = np.array(cache._host_lens)
    scores = dec.scores.cpu().numpy().astype(np.float64)
    ids = dec.ids.cpu().numpy().astype(np.int64)
    n_b = (lens + page - 1) // page
    # selection: bit-exact on the kernel's fp32 scores, per batch (ragged page counts)
    for bi in range(b):
        kb = max(1, min(topk, n_b[bi]))
        want = oracle.topk_lowest_index(scores[bi, :, :, : n_b[bi]], kb)
        assert np.array_equal(ids[bi, :, :, :kb], want)
    # metadata (outward-rounded for narrow meta) and scores vs the oracle
    kp = _np(cache.k_pool)
    if cache.fp8:
        kp = kp * cache.k_scale.cpu().numpy()[:, :, None, None]
    vp = _np(cache.v_pool)
    if cache.fp8:
        vp = vp * cache.v_scale.cpu().numpy()[:, :, None, None]
    mm, mx = _np(cache.meta_min), _np(cache.meta_max)  # (B, H_kv, max_pages, D), logical pages
    for bi in range(b):
        for p in range(n_b[bi]):
            phys = int(table[bi, p])
            rows = min(page, lens[bi] - p * page)
            assert np.all(mm[bi, :, p] <= kp[phys, :, :rows].min(axis=1))
            assert np.all(mx[bi, :, p] >= kp[phys, :, :rows].max(axis=1))
    # union lists + attention over them vs the oracle
    group = hq // hkv
    cnt = dec.union_count.cpu().numpy()[:, :, 0]
    uids = dec.union_ids.cpu().numpy()[:, :, 0]
    for bi in range(b):
        kb = max(1, min(topk, n_b[bi]))
        union = oracle.gqa_union(ids[bi:bi + 1, :, :, :kb], int(n_b[bi]), group)[0, :, 0]
        for kh in range(hkv):
            assert np.array_equal(uids[bi, kh, : cnt[bi, kh]], np.nonzero(union[kh])[0])
    ref = oracle.paged_sparse_decode(_np(q)[:, :, 0], kp, vp, table.numpy(), lens, uids, cnt, page_size=page)
    assert_close_16(out[:, :, 0], ref, tol)
    return dec, out


def test_quest_decode_config1_shape(cuda):
    """Config 1: B=1, H_q=32, H_kv=8, D=128, T=4096, pages of 16, top-32 pages, fp16,
    2% needle pages along a query direction."""
    gen = torch.Generator().manual_seed(1)
    b, hq, hkv, d, page, t = 1, 32, 8, 128, 16, 4096
    q = torch.randn(b, hq, 1, d, generator=gen)
    dirs = torch.nn.functional.normalize(q[0, ::4, 0], dim=-1)  # one direction per kv head
    cache, table = _make_paged(b, hkv, d, page, [t], torch.float16, gen, needles=0.02, q_dirs=dirs, perm=False)
    _check_decode(cache, table, q.half().to(cuda), 32, 0, TOL_16)


@pytest.mark.parametrize("lens", [[8192, 8192, 8192, 8192], [8192, 5000, 64, 6401]])
def test_quest_decode_config2_shape_reduced(cuda, lens):
    """Config 2 layout (bf16, pages of 64, 32 + sink + last, permuted pool), reduced T,
    including ragged sequence lengths."""
    gen = torch.Generator().manual_seed(sum(lens))
    b, hq, hkv, d, page = len(lens), 32, 8, 128, 64
    q = torch.randn(b, hq, 1, d, generator=gen)
    cache, table = _make_paged(b, hkv, d, page, lens, torch.bfloat16, gen)
    _check_decode(cache, table, q.to(torch.bfloat16).to(cuda), 34, 1, TOL_16)


@pytest.mark.parametrize("chunks", [1, 2, 3, 7])
def test_quest_decode_select_chunks(cuda, chunks):
    """The single-CTA fused selection (1 chunk) and the candidates form + merge (several
    chunks, ragged sequences ending inside and before chunks) give the same top-k, union
    and output."""
    gen = torch.Generator().manual_seed(100 + chunks)
    lens = [8192, 5000, 64, 6401, 8129]
    b, hq, hkv, d, page = len(lens), 16, 2, 128, 64
    q = torch.randn(b, hq, 1, d, generator=gen)
    cache, table = _make_paged(b, hkv, d, page, lens, torch.bfloat16, gen)
    _check_decode(cache, table, q.to(torch.bfloat16).to(cuda), 34, 1, TOL_16, chunks=chunks)


def test_paged_bad_page_id_reports_status(cuda, monkeypatch):
    """A page-table entry outside the pool is skipped and reported, never read."""
    from linattn_b200 import QuestDecoder, _lib as L

    monkeypatch.setenv("LINATTN_B200_STRICT", "0")

    gen = torch.Generator().manual_seed(5)
    cache, table = _make_paged(1, 2, 64, 16, [256], torch.float16, gen)
    dec = QuestDecoder(cache, 4, 4)
    q = torch.randn(1, 4, 1, 64, device=cuda, dtype=torch.float16)
    L.read_status(cache.device)
    cache.page_table[0, 3] = cache.num_phys_pages + 5  # past the pool
    dec.step(q)
    bits = L.read_status(cache.device)
    assert bits & L.DEV_BAD_ID


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bs", [1, 16, 48, 128])
def test_block_sparse_page_sizes(cuda, dtype, bs):
    """Per-token lists (block 1, the DSA form), blocks smaller than, not dividing, and
    larger than a warp tile; -1 padding in the lists."""
    from linattn_b200 import block_sparse_attention

    gen = torch.Generator().manual_seed(bs)
    b, hq, hkv, tq, tk, d = 2, 8, 2, 4, 700, 128
    n_blocks = (tk + bs - 1) // bs
    n = min(n_blocks, 300 if bs == 1 else 9)
    q = torch.randn(b, hq, tq, d, generator=gen).to(dtype)
    k = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    v = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    ids = torch.stack([torch.randperm(n_blocks, generator=gen)[:n] for _ in range(b * hkv * tq)]).view(b, hkv, tq, n)
    ids[..., -2:] = -1  # padding
    out = block_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), ids.to(cuda), block_size=bs)
    ref = oracle.block_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                        np.where(ids.numpy() < 0, 10 ** 9, ids.numpy()), block_size=bs)
    assert_close_16(out, ref)


@pytest.mark.parametrize("union", [True, False])
def test_cuda_quest_variant_bf16_d128_chunked(cuda, union):
    """Chunked prefill + decode through cuda_quest at the BASELINE head size (the
    tensor-core path with the causal limit inside pages)."""
    from linattn_b200 import AttnConfig, build

    gen = torch.Generator().manual_seed(5)
    b, hq, hkv, t, d, page, topk = 2, 8, 2, 700, 128, 16, 7
    q = torch.randn(b, hq, t, d, generator=gen).to(torch.bfloat16)
    k = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16)
    v = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16)
    cfg = AttnConfig(n_heads=hq, n_kv_heads=hkv, head_dim=d, block_size=page, topk_blocks=topk,
                     extras={} if union else {"gqa_union": False})
    out, _ = build("cuda_quest", cfg).forward(q.to(cuda), k.to(cuda), v.to(cuda), chunk=256)
    qf, kf, vf = (x.float().numpy() for x in (q, k, v))
    outs, ambiguous = [], []
    group = hq // hkv
    for start in range(0, t, 256):
        qc = qf[:, :, start:start + 256]
        kc, vc = kf[:, :, : start + 256], vf[:, :, : start + 256]
        mask = oracle.quest_effective_mask(qc, kc, page, topk, offset=start, group=group, gqa_union_mode=union)
        outs.append(oracle.dense_attention(qc, kc, vc, mask=mask))
        # rows whose k-th and (k+1)-th float64 page bounds are within 1e-2: the kernel's
        # fp32 sums may legitimately pick the other page there
        mins, maxs = oracle.page_bounds(kc, page)
        _, sc = oracle.page_select(qc, mins, maxs, page, topk, offset=start)
        srt = -np.sort(-np.where(np.isfinite(sc), sc, np.where(sc > 0, 1e30, -1e30)), axis=-1)
        kk = min(topk, sc.shape[-1])
        gap = np.abs(srt[..., kk - 1] - srt[..., kk]) if kk < sc.shape[-1] else np.full(sc.shape[:-1], np.inf)
        gap = np.where(srt[..., min(kk, sc.shape[-1] - 1)] > -1e29, gap, np.inf)  # < k+1 visible: no choice
        amb = gap < 1e-2
        if union:
            amb = np.repeat(amb.reshape(b, hkv, group, -1).any(2), group, axis=1)
        ambiguous.append(amb)
    ref = np.concatenate(outs, axis=2)
    amb = np.concatenate(ambiguous, axis=2)
    got = out.float().cpu().numpy()
    ok = np.all(np.abs(got - ref) <= TOL_16 + 2.0 ** -8 * np.abs(ref), axis=-1)
    assert amb.mean() < 0.1  # the check must cover most rows
    assert np.all(ok | amb), f"{int((~ok & ~amb).sum())} unambiguous rows differ"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rows_past_sequence_end_are_never_used(cuda, dtype):
    """K/V views into a larger buffer whose rows past T_k hold NaN: the tail page's
    box brings those rows in, and the result must still be the oracle's."""
    from linattn_b200 import block_sparse_attention

    gen = torch.Generator().manual_seed(9)
    b, hq, hkv, tq, tk, t_alloc, d, bs = 2, 8, 2, 3, 700, 1024, 128, 64
    kbuf = torch.full((b, hkv, t_alloc, d), float("nan"), dtype=dtype)
    vbuf = torch.full((b, hkv, t_alloc, d), float("nan"), dtype=dtype)
    kbuf[:, :, :tk] = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    vbuf[:, :, :tk] = torch.randn(b, hkv, tk, d, generator=gen).to(dtype)
    q = torch.randn(b, hq, tq, d, generator=gen).to(dtype)
    ids = torch.tensor([10, 3, 0, 7]).view(1, 1, 1, 4).expand(b, hkv, tq, 4).contiguous()  # 10 = the tail page
    kd, vd = kbuf.to(cuda), vbuf.to(cuda)
    out = block_sparse_attention(q.to(cuda), kd[:, :, :tk], vd[:, :, :tk], ids.to(cuda), block_size=bs)
    k, v = kbuf[:, :, :tk], vbuf[:, :, :tk]
    ref = oracle.block_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), ids.numpy(),
                                        block_size=bs)
    assert torch.isfinite(out).all()
    assert_close_16(out, ref)


def test_quest_decode_fp8_kv(cuda):
    """Config-5 storage: fp8 e4m3 KV with one fp32 scale per (page, kv head), GQA 8.
    Output within 1e-2 of the fp32 oracle on the dequantised KV with the kernel's own
    selection; the quantisation error against the unquantised KV is only reported."""
    from linattn_b200 import PagedKVCache, QuestDecoder
    from oracle.quant import dequantize_fp8, quantize_fp8

    gen = torch.Generator().manual_seed(55)
    b, hq, hkv, d, page, t, topk = 2, 16, 2, 128, 64, 64 * 48, 12
    k = torch.randn(b, hkv, t, d, generator=gen)
    v = torch.randn(b, hkv, t, d, generator=gen)
    q = torch.randn(b, hq, 1, d, generator=gen).to(torch.bfloat16)
    cache = PagedKVCache(b, hkv, d, page, t // page, dtype=torch.float8_e4m3fn, device="cuda")
    table = torch.randperm(b * (t // page), generator=gen).view(b, t // page).to(torch.int32)
    lens = [t, t - 77]
    cache.fill(k.to(cuda), v.to(cuda), lens, table)
    dec = QuestDecoder(cache, hq, topk, sink_pages=1, keep_scores=True)
    out = dec.step(q.to(cuda))
    torch.cuda.synchronize()
    # codec parity: the kernel-side pool equals the oracle codec (kv/quant.py) per page and head
    kp = k.view(b, hkv, t // page, page, d).transpose(1, 2).numpy()
    codes, scale = quantize_fp8(kp, reduce_axes=(3, 4))
    got_codes = cache.k_pool[table.long().view(-1)].view(b, t // page, hkv, page, d).cpu().numpy()
    assert np.array_equal(got_codes, codes)
    got_scale = cache.k_scale[table.long().view(-1)].view(b, t // page, hkv).cpu().numpy()
    assert np.array_equal(got_scale, scale.reshape(b, t // page, hkv))
    kdq = dequantize_fp8(codes, scale)  # (b, n, hkv, P, D)
    vcodes, vscale = quantize_fp8(v.view(b, hkv, t // page, page, d).transpose(1, 2).numpy(), reduce_axes=(3, 4))
    vdq = dequantize_fp8(vcodes, vscale)
    n_phys = b * (t // page)
    kpool = np.zeros((n_phys, hkv, page, d), np.float32)
    vpool = np.zeros_like(kpool)
    for bi in range(b):
        for pg in range(t // page):
            kpool[table[bi, pg]] = kdq[bi, pg]
            vpool[table[bi, pg]] = vdq[bi, pg]
    cnt = dec.union_count.cpu().numpy()[:, :, 0]
    uids = dec.union_ids.cpu().numpy()[:, :, 0]
    ref = oracle.paged_sparse_decode(_np(q)[:, :, 0], kpool, vpool, table.numpy(), np.array(lens), uids, cnt,
                                     page_size=page)
    assert_close_16(out[:, :, 0], ref, tol=1e-2)
    # metadata bounds the dequantised keys (rounded outward to bf16)
    mm, mx = _np(cache.meta_min), _np(cache.meta_max)
    for bi in range(b):
        for pg in range(-(-lens[bi] // page)):
            rows = min(page, lens[bi] - pg * page)
            assert np.all(mm[bi, :, pg] <= kdq[bi, pg, :, :rows].min(axis=1))
            assert np.all(mx[bi, :, pg] >= kdq[bi, pg, :, :rows].max(axis=1))
    # selection bit-exact on the kernel's own scores
    scores = dec.scores.cpu().numpy().astype(np.float64)
    ids = dec.ids.cpu().numpy()
    for bi in range(b):
        nb = -(-lens[bi] // page)
        assert np.array_equal(ids[bi, :, :, :topk], oracle.topk_lowest_index(scores[bi, :, :, :nb], topk))
