"""Decode / chunk append into the paged pool (``linattn_paged_append`` through
``PagedKVCache.append``): the new rows land at their positions through the page table,
converted to the pool dtype, and the bounds of every touched page equal the oracle's
page bounds of the whole sequence (``QuestAttention._refresh_pages``,
src/linattn/variants/selection.py:181-201), bit for bit when the metadata has the
keys' dtype, and equal to a full recomputation (``refresh_meta``) when it is narrower.
Cases: empty and partly filled starting pages, appends that cross page boundaries and
map new pages from the allocator, 1-token decode steps and longer chunks."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _pool_rows(cache, b, n):
    """Rows [0, n) of sequence b as (H_kv, n, D) float64, read through the page table."""
    p = cache.page_size
    table = cache.page_table[b].long().cpu()
    pos = torch.arange(n)
    phys = table[pos // p]
    k = cache.k_pool.cpu()[phys, :, pos % p].transpose(0, 1)
    v = cache.v_pool.cpu()[phys, :, pos % p].transpose(0, 1)
    return k.double().numpy(), v.double().numpy()


@pytest.mark.parametrize("pool,meta,src", [(torch.bfloat16, None, torch.bfloat16), (torch.float16, None, torch.float32),
                                           (torch.float32, None, torch.float32),
                                           (torch.float32, torch.bfloat16, torch.float32)])
def test_append_rows_and_bounds(cuda, pool, meta, src):
    from linattn_b200 import PagedKVCache

    gen = torch.Generator().manual_seed(11)
    b, hkv, d, p, max_pages = 4, 2, 128, 64, 12
    init = [0, 63, 64, 130]
    cache = PagedKVCache(b, hkv, d, p, max_pages, num_phys_pages=b * max_pages, dtype=pool, meta_dtype=meta,
                         device="cuda")
    k0 = torch.randn(b, hkv, max(init), d, generator=gen)
    v0 = torch.randn(b, hkv, max(init), d, generator=gen)
    table = torch.randperm(b * max_pages, generator=gen).view(b, max_pages).to(torch.int32)
    cache.fill(k0.to(cuda), v0.to(cuda), init, table)
    full_k = [k0[i, :, : init[i]].to(pool).double() for i in range(b)]
    full_v = [v0[i, :, : init[i]].to(pool).double() for i in range(b)]
    for tn in (1, 5, 64, 1, 100):
        kn = torch.randn(b, hkv, tn, d, generator=gen).to(src)
        vn = torch.randn(b, hkv, tn, d, generator=gen).to(src)
        cache.append(kn.to(cuda), vn.to(cuda))
        torch.cuda.synchronize()
        for i in range(b):
            full_k[i] = torch.cat([full_k[i], kn[i].to(pool).double()], dim=1)
            full_v[i] = torch.cat([full_v[i], vn[i].to(pool).double()], dim=1)
        lens = cache.seq_lens.cpu().tolist()
        for i in range(b):
            n = full_k[i].shape[1]
            assert lens[i] == n
            gk, gv = _pool_rows(cache, i, n)
            assert np.array_equal(gk, full_k[i].numpy())
            assert np.array_equal(gv, full_v[i].numpy())
            mins, maxs = oracle.page_bounds(full_k[i].numpy()[None], p)
            npg = mins.shape[2]
            got_min = cache.meta_min[i, :, :npg].double().cpu().numpy()
            got_max = cache.meta_max[i, :, :npg].double().cpu().numpy()
            if meta is None or meta == pool:
                assert np.array_equal(got_min, mins[0])
                assert np.array_equal(got_max, maxs[0])
            else:
                assert np.all(got_min <= mins[0]) and np.all(got_max >= maxs[0])
    if meta is not None and meta != pool:
        # narrower metadata: identical to a recomputation over every row of every page
        folded = cache.meta.clone()
        cache.refresh_meta()
        torch.cuda.synchronize()
        assert torch.equal(folded, cache.meta)


def test_append_decode_steps_match_refresh(cuda):
    """Forty 1-token steps (crossing a page boundary) then a full recomputation: the
    incrementally folded bounds are unchanged by it."""
    from linattn_b200 import PagedKVCache

    gen = torch.Generator().manual_seed(12)
    b, hkv, d, p = 3, 8, 128, 16
    cache = PagedKVCache(b, hkv, d, p, 16, dtype=torch.bfloat16, device="cuda")
    k0 = torch.randn(b, hkv, 40, d, generator=gen).to(torch.bfloat16)
    cache.fill(k0.to(cuda), k0.to(cuda), [40, 7, 33])
    for _ in range(40):
        kn = torch.randn(b, hkv, 1, d, generator=gen).to(torch.bfloat16).to(cuda)
        cache.append(kn, -kn)
    torch.cuda.synchronize()
    assert cache.seq_lens.cpu().tolist() == [80, 47, 73]
    folded = cache.meta.clone()
    cache.refresh_meta()
    torch.cuda.synchronize()
    assert torch.equal(folded, cache.meta)


def test_append_fp8_pool_refused(cuda):
    from linattn_b200 import PagedKVCache

    cache = PagedKVCache(1, 1, 128, 64, 2, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(NotImplementedError):
        cache.append(torch.zeros(1, 1, 1, 128, device=cuda), torch.zeros(1, 1, 1, 128, device=cuda))
