"""Sequence-sharded Quest decode (the million-token configuration) emulated on one GPU.

R shard caches hold contiguous page ranges of every sequence; the all-gathers are
stacks.  The merged global selection must equal the single-cache decoder's selection
bit for bit (same metadata, same fp32 scores, lowest-page ties), and the combined output
the oracle's attention over the union of the selected pages.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def _build(dtype, b, hkv, d, page, n_pages, world, gen):
    from linattn_b200 import PagedKVCache
    from linattn_b200.sharded import shard_page_ranges

    t = n_pages * page
    k = torch.randn(b, hkv, t, d, generator=gen)
    v = torch.randn(b, hkv, t, d, generator=gen)
    full = PagedKVCache(b, hkv, d, page, n_pages, dtype=dtype, device="cuda")
    full.fill(k.cuda(), v.cuda(), [t] * b)
    shards = []
    for r in range(world):
        lo, hi = shard_page_ranges(n_pages, world, r)
        c = PagedKVCache(b, hkv, d, page, hi - lo, dtype=dtype, device="cuda")
        c.fill(k[:, :, lo * page:hi * page].cuda(), v[:, :, lo * page:hi * page].cuda(), [(hi - lo) * page] * b)
        shards.append((c, lo, hi))
    return full, shards, k, v


@pytest.mark.parametrize("dtype,world", [(torch.bfloat16, 3), (torch.float8_e4m3fn, 2), (torch.bfloat16, 1)])
def test_sharded_decode_matches_single_cache(cuda, dtype, world):
    from linattn_b200 import QuestDecoder
    from linattn_b200.sharded import ShardedQuestDecoder

    gen = torch.Generator().manual_seed(7 + world)
    b, hq, hkv, d, page, n_pages, topk, sink = 2, 16, 2, 128, 64, 40, 8, 1
    full, shards, k, v = _build(dtype, b, hkv, d, page, n_pages, world, gen)
    q = torch.randn(b, hq, 1, d, generator=gen).bfloat16().cuda()
    ref_dec = QuestDecoder(full, hq, topk, sink_pages=sink, keep_scores=True)
    ref_out = ref_dec.step(q)
    decs = [ShardedQuestDecoder(c, hq, topk, [lo] * b, [hi] * b, sink_pages=sink, last_here=(hi == n_pages),
                                sink_here=(lo == 0), n_ranks=world) for c, lo, hi in shards]
    cands = [dec.candidates(q) for dec in decs]
    all_s = torch.stack([c[0] for c in cands]).flatten(0, 1)  # (R * chunks, B, H_q, K)
    all_i = torch.stack([c[1] for c in cands]).flatten(0, 1)
    for dec in decs:
        dec.merge(all_s, all_i)
    parts = [dec.partial(q) for dec in decs]
    all_o = torch.stack([p[0].reshape(-1, d) for p in parts])
    all_l = torch.stack([p[1].reshape(-1) for p in parts])
    out = decs[0].combine(all_o, all_l)
    torch.cuda.synchronize()
    # the global selection equals the single cache's, order included
    ref_ids = ref_dec.ids[:, :, 0].cpu().numpy()
    for dec in decs:
        assert np.array_equal(dec.sel.cpu().numpy(), ref_ids)
    # every shard's union is the single-cache union restricted to its pages
    ref_cnt = ref_dec.union_count[:, :, 0].cpu().numpy()
    ref_u = ref_dec.union_ids[:, :, 0].cpu().numpy()
    for dec, (c, lo, hi) in zip(decs, shards):
        cnt = dec.union_count[:, :, 0].cpu().numpy()
        u = dec.union_ids[:, :, 0].cpu().numpy()
        for bi in range(b):
            for kh in range(hkv):
                want = [x - lo for x in ref_u[bi, kh, :ref_cnt[bi, kh]] if lo <= x < hi]
                assert list(u[bi, kh, :cnt[bi, kh]]) == want
    # output: the oracle's attention over the single-cache union (dequantised pages)
    if full.fp8:  # e4m3 codes x per-(page, kv head) scales
        kp = oracle.e4m3_decode(full.k_pool.cpu().numpy()) * full.k_scale.cpu().numpy()[:, :, None, None]
        vp = oracle.e4m3_decode(full.v_pool.cpu().numpy()) * full.v_scale.cpu().numpy()[:, :, None, None]
    else:
        kp, vp = _np(full.k_pool), _np(full.v_pool)
    ref = oracle.paged_sparse_decode(_np(q)[:, :, 0], kp, vp, full.page_table.cpu().numpy(),
                                     np.array([n_pages * page] * b), ref_u, ref_cnt, page_size=page)
    tol = 1e-2 if full.fp8 else 2e-3
    err = np.abs(_np(out[:, :, 0]) - ref)
    assert np.all(err <= tol + 2.0 ** -8 * np.abs(ref)), err.max()
    # and the single-cache decoder agrees with it too
    assert np.abs(_np(ref_out[:, :, 0]) - ref).max() <= tol + 2.0 ** -8 * np.abs(ref).max()


@pytest.mark.parametrize("world,chunks", [(1, None), (1, 5), (2, None), (2, 3), (4, 2)])
def test_sharded_decode_packed_exchange(cuda, world, chunks):
    """The packed path of ``step``: one gathered [scores | ids] buffer and one gathered
    [o | lse] buffer per rank, read in place by the merge and combine kernels through
    their rank strides; several chunks per shard (merged by the shard before the
    exchange when there are several ranks)."""
    from linattn_b200 import QuestDecoder
    from linattn_b200.sharded import ShardedQuestDecoder

    gen = torch.Generator().manual_seed(31 + world)
    b, hq, hkv, d, page, n_pages, topk = 3, 8, 2, 128, 64, 36, 6
    full, shards, k, v = _build(torch.bfloat16, b, hkv, d, page, n_pages, world, gen)
    q = torch.randn(b, hq, 1, d, generator=gen).bfloat16().cuda()
    ref_dec = QuestDecoder(full, hq, topk, keep_scores=True)
    ref_out = ref_dec.step(q).clone()
    decs = [ShardedQuestDecoder(c, hq, topk, [lo] * b, [hi] * b, last_here=(hi == n_pages), sink_here=(lo == 0),
                                n_ranks=world, select_chunks=chunks) for c, lo, hi in shards]
    if world == 1:
        out = decs[0].step(q, exchange=lambda t: t.unsqueeze(0))
    else:
        for dec in decs:
            dec.candidates(q)
        # each rank exchanges one sorted block of K per head once it merged its chunks
        assert all(dec.premerge == (dec.chunks > 1) for dec in decs)
        allc = torch.stack([dec.exchange_buf for dec in decs])
        for dec in decs:
            dec.merge_packed(allc)
        for dec in decs:
            dec.partial(q)
        out = decs[0].combine_packed(torch.stack([dec.part for dec in decs]))
    torch.cuda.synchronize()
    ref_ids = ref_dec.ids[:, :, 0].cpu().numpy()
    for dec in decs:
        assert np.array_equal(dec.sel.cpu().numpy(), ref_ids)
    err = (out.float() - ref_out.float()).abs().max().item()
    assert err <= 2e-3 + 2.0 ** -8 * ref_out.float().abs().max().item(), err
