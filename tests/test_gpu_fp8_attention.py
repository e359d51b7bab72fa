"""fp8 e4m3 paged sparse attention (one fp32 scale per (page, kv head)) against the
fp64 oracle on the dequantised codes: outputs within 1e-2 max-abs, lse within 1e-3.

D = 128 with pages of >= 32 rows and a 16-bit q runs the tensor-core kernel (codes to
f16 in registers); pages of 16 rows, D = 64 and an fp32 q run the CUDA-core kernel.
Cases cover
ragged sequence ends (partial tiles), pages of 48 rows (a tile reaching past the page),
GQA groups of 4, 6, 8 and 16 (two head chunks), -1 list entries, split-KV, f16 / f32
queries, f32 outputs with lse, zero-scale pages and causal multi-query rows."""
import math

import numpy as np
import pytest
import torch

import oracle
from oracle.quant import e4m3_decode

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _fp8_cache(b, hkv, d, page, lens, gen, *, zero_k=(), zero_v=(), needle_dir=None):
    """Paged fp8 cache with a random page table; codes from N(0,1) rows quantised per
    (page, kv head); `zero_k` / `zero_v` list physical pages whose scale is 0."""
    from linattn_b200 import PagedKVCache

    max_pages = max(-(-x // page) for x in lens)
    n_phys = b * max_pages
    cache = PagedKVCache(b, hkv, d, page, max_pages, num_phys_pages=n_phys, dtype=torch.float8_e4m3fn,
                         device="cuda")
    host = {}
    for name, zero in (("k", zero_k), ("v", zero_v)):
        x = torch.randn(n_phys, hkv, page, d, generator=gen)
        if name == "k" and needle_dir is not None:
            x[: max(1, n_phys // 20)] += 2.0 * needle_dir
        sc = x.abs().amax(dim=(2, 3)).clamp_min(1e-8) / 448.0
        codes = (x / sc[:, :, None, None]).to(torch.float8_e4m3fn).view(torch.uint8)
        for p in zero:
            sc[p] = 0.0
        getattr(cache, f"{name}_pool").copy_(codes)
        getattr(cache, f"{name}_scale").copy_(sc)
        host[name] = (e4m3_decode(codes.numpy()).astype(np.float64), sc.numpy().astype(np.float64))
    table = torch.randperm(n_phys, generator=gen).view(b, max_pages).to(torch.int32)
    cache.set_page_table(table, lens)
    return cache, table.numpy(), host


def _lists(b, hkv, n_pages, n, gen, *, holes=False):
    ids = torch.stack([torch.stack([torch.randperm(n_pages, generator=gen)[:n] for _ in range(hkv)])
                       for _ in range(b)]).to(torch.int32)
    if holes:
        ids[:, :, ::5] = -1
    counts = torch.randint(max(1, n // 2), n + 1, (b, hkv), generator=gen).to(torch.int32)
    return ids, counts


def _run(cuda, q, cache, ids, counts, *, causal=False, offset=0, n_splits=None, out_dtype=None, lse=True):
    from linattn_b200.block_sparse import lists_desc, sparse_attention

    b, hq, tq, d = q.shape
    qd = q.to(cuda)
    ids_d, counts_d = ids.to(cuda), counts.to(cuda)
    out = torch.empty(qd.shape, dtype=out_dtype or q.dtype, device=cuda)
    lse_out = torch.empty(b, hq, tq, dtype=torch.float32, device=cuda) if lse else None
    sparse_attention(qd, cache.kv_desc(), lists_desc(ids_d, cache.n_kv_heads, counts_d), causal=causal, offset=offset,
                     out=out, lse_out=lse_out, n_splits=n_splits)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), (lse_out.cpu().numpy() if lse else None)


def _reference(q, table, lens, ids, counts, host, page, *, causal=False, offset=0):
    qn = q.float().numpy().astype(np.float64)
    b, hq, tq, d = qn.shape
    (kc, ks), (vc, vs) = host["k"], host["v"]
    # a -1 list entry selects nothing: drop them (the oracle takes every listed id)
    ids_np, cnt_np = ids.numpy(), counts.numpy()
    kept = np.full_like(ids_np, 0)
    kept_n = np.zeros_like(cnt_np)
    for bi in range(ids_np.shape[0]):
        for h in range(ids_np.shape[1]):
            row = ids_np[bi, h, : cnt_np[bi, h]]
            row = row[row >= 0]
            kept[bi, h, : row.size] = row
            kept_n[bi, h] = row.size
    ids, counts = torch.from_numpy(kept), torch.from_numpy(kept_n)
    out = np.zeros((b, hq, tq, d))
    lse = np.zeros((b, hq, tq))
    for t in range(tq):
        qpos = np.full(b, offset + t) if causal else None
        o, l = oracle.paged_sparse_decode(qn[:, :, t], kc, vc, table, np.array(lens), ids.numpy(), counts.numpy(),
                                          page_size=page, k_scale=ks, v_scale=vs, q_pos=qpos, return_lse=True)
        out[:, :, t], lse[:, :, t] = o, l
    return out, lse


def _check(got, want, got_lse=None, want_lse=None):
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    assert err < TOL, f"max abs err {err}"
    if got_lse is not None:
        fin = np.isfinite(want_lse)
        assert np.array_equal(np.isfinite(got_lse), fin)
        assert np.abs(got_lse[fin] - want_lse[fin]).max() < 1e-3


@pytest.mark.parametrize("page", [32, 48, 64, 128, 16])
@pytest.mark.parametrize("group", [8, 4])
def test_fp8_decode_pages(cuda, page, group):
    gen = torch.Generator().manual_seed(100 + page + group)
    b, hkv, d = 3, 2, 128
    n_pages = 24
    lens = [n_pages * page, n_pages * page - 5, 7 * page + 3]
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen)
    ids, counts = _lists(b, hkv, n_pages, 14, gen)
    q = torch.randn(b, hkv * group, 1, d, generator=gen).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    _check(got, want, got_lse, want_lse)


@pytest.mark.parametrize("group,splits", [(6, 1), (16, 1), (8, 3), (16, 4)])
def test_fp8_decode_groups_and_splits(cuda, group, splits):
    gen = torch.Generator().manual_seed(200 + group * 10 + splits)
    b, hkv, d, page = 2, 2, 128, 64
    n_pages = 40
    lens = [n_pages * page - 9, 30 * page]
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen)
    ids, counts = _lists(b, hkv, n_pages, 33, gen, holes=True)
    q = torch.randn(b, hkv * group, 1, d, generator=gen).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts, n_splits=splits)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    _check(got, want, got_lse, want_lse)


@pytest.mark.parametrize("qdtype,odtype", [(torch.float16, torch.float16), (torch.float32, torch.float32),
                                           (torch.bfloat16, torch.float32)])
def test_fp8_decode_q_and_out_dtypes(cuda, qdtype, odtype):
    gen = torch.Generator().manual_seed(300)
    b, hkv, d, page, group = 2, 2, 128, 64, 8
    n_pages = 16
    lens = [n_pages * page, 11 * page - 1]
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen)
    ids, counts = _lists(b, hkv, n_pages, 12, gen)
    # wide dynamic range across heads (the per-head power-of-two q factor)
    q = torch.randn(b, hkv * group, 1, d, generator=gen) * torch.logspace(-3, 2, hkv * group).view(1, -1, 1, 1)
    q = q.to(qdtype)
    got, got_lse = _run(cuda, q, cache, ids, counts, out_dtype=odtype)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    scale = np.maximum(1.0, np.abs(want).max(axis=-1, keepdims=True))
    _check(got / scale, want / scale)
    fin = np.isfinite(want_lse)
    assert np.abs(got_lse[fin] - want_lse[fin]).max() < 1e-3 * max(1.0, np.abs(want_lse[fin]).max())


def test_fp8_zero_scale_pages(cuda):
    """A page whose K scale is 0 scores 0 (it still takes softmax mass); one whose V
    scale is 0 contributes a zero value."""
    gen = torch.Generator().manual_seed(400)
    b, hkv, d, page, group = 2, 2, 128, 64, 8
    n_pages = 12
    lens = [n_pages * page] * b
    n_phys = b * n_pages
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen, zero_k=range(0, n_phys, 3),
                                    zero_v=range(1, n_phys, 4))
    ids, counts = _lists(b, hkv, n_pages, 10, gen)
    q = torch.randn(b, hkv * group, 1, d, generator=gen).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    _check(got, want, got_lse, want_lse)


@pytest.mark.parametrize("offset", [0, 700])
def test_fp8_causal_queries(cuda, offset):
    gen = torch.Generator().manual_seed(500 + offset)
    b, hkv, d, page, group, tq = 2, 2, 128, 32, 4, 3
    n_pages = 40
    lens = [n_pages * page] * b
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen)
    ids = torch.stack([torch.stack([torch.arange(n_pages) for _ in range(hkv)]) for _ in range(b)]).to(torch.int32)
    counts = torch.full((b, hkv), n_pages, dtype=torch.int32)
    q = torch.randn(b, hkv * group, tq, d, generator=gen).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts, causal=True, offset=offset)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page, causal=True, offset=offset)
    _check(got, want, got_lse, want_lse)


def test_fp8_d64_runs_cuda_core_path(cuda):
    gen = torch.Generator().manual_seed(600)
    b, hkv, d, page, group = 2, 2, 64, 64, 4
    n_pages = 10
    lens = [n_pages * page, 5 * page + 17]
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen)
    ids, counts = _lists(b, hkv, n_pages, 8, gen)
    q = torch.randn(b, hkv * group, 1, d, generator=gen).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    _check(got, want, got_lse, want_lse)


def test_fp8_needles_dominate(cuda):
    """Keys with a strong q-aligned component: large scores (the softmax maximum moves
    from tile to tile across pages of different K scales)."""
    gen = torch.Generator().manual_seed(700)
    b, hkv, d, page, group = 2, 2, 128, 64, 8
    n_pages = 32
    lens = [n_pages * page] * b
    u = torch.nn.functional.normalize(torch.randn(d, generator=gen), dim=0) * math.sqrt(d)
    cache, table, host = _fp8_cache(b, hkv, d, page, lens, gen, needle_dir=u)
    ids, counts = _lists(b, hkv, n_pages, 32, gen)
    q = (u + 0.5 * torch.randn(b, hkv * group, 1, d, generator=gen)).to(torch.bfloat16)
    got, got_lse = _run(cuda, q, cache, ids, counts)
    want, want_lse = _reference(q, table, lens, ids, counts, host, page)
    _check(got, want, got_lse, want_lse)
