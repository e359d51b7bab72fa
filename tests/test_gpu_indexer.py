"""GPU parity of the lightning indexer + top-k (``indexer_topk``) against the oracle.

Scores are fp32 sums in a different order than the float64 oracle, so they are checked
within a relative tolerance; the selection is checked bit-exact against the oracle's
lowest-index top-k applied to the kernel's own fp32 scores (the "identical fp32
scores" criterion), and against the reference's golden vectors.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle.quest import topk_lowest_index
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy() if t.dtype != torch.float64 else t.cpu().numpy()


def _inputs(b, tq, tk, h, d, seed, dtype=torch.float32, w_scale=1.0 / 8):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, tq, h, d, generator=g).to(dtype)
    k = torch.randn(b, tk, h, d, generator=g).to(dtype)
    w = (torch.randn(b, tq, h, generator=g) * w_scale).to(dtype)
    return q, k, w


def _check_selection_on_own_scores(scores, vals, idx, kk, causal=False, offset=0):
    """Selection bit-exact on the kernel's fp32 scores (lowest index first on ties)."""
    s = _np(scores).astype(np.float64)
    tq, tk = s.shape[1], s.shape[2]
    if causal:
        allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + offset)
        s = np.where(allow[None], s, -np.inf)
    ref_idx = topk_lowest_index(s, kk)
    ref_vals = np.take_along_axis(s, ref_idx, axis=-1)
    if causal:
        ref_idx = np.where(np.isneginf(ref_vals), -1, ref_idx)
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    assert np.array_equal(_np(vals).astype(np.float64), ref_vals)


def test_indexer_golden(cuda):
    from linattn_b200 import indexer_topk

    g = golden("indexer")
    vals, idx = indexer_topk(torch.from_numpy(g["q"]).to(cuda), torch.from_numpy(g["k"]).to(cuda),
                             torch.from_numpy(g["w"]).to(cuda), int(g["topk"]))
    assert idx.dtype == torch.int64 and vals.dtype == torch.float32
    assert np.allclose(_np(vals), g["vals"], atol=1e-5)
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    vals2, idx2 = indexer_topk(torch.from_numpy(g["q2"]).to(cuda), torch.from_numpy(g["k2"]).to(cuda),
                               torch.from_numpy(g["w2"]).to(cuda), int(g["topk2"]))
    assert np.allclose(_np(vals2), g["vals2"], atol=1e-5)
    # near-ties may legitimately reorder; the sets must agree outside a 1e-5 band
    s = oracle.indexer_scores(g["q2"], g["k2"], g["w2"])
    kth = np.sort(s, -1)[..., ::-1][..., int(g["topk2"]) - 1:int(g["topk2"])]
    for a, b_, row_s, kv in zip(idx2.cpu().numpy().reshape(-1, 10), g["idx2"].reshape(-1, 10),
                                s.reshape(-1, s.shape[-1]), kth.reshape(-1)):
        clear = set(np.nonzero(row_s > kv + 1e-5)[0])
        assert clear <= set(a.tolist()) and clear <= set(b_.tolist())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,tq,tk,h,d,k", [(1, 40, 300, 4, 64, 32), (2, 33, 129, 3, 8, 7), (1, 5, 64, 1, 16, 64)])
def test_indexer_scores_and_selection(cuda, dtype, b, tq, tk, h, d, k):
    from linattn_b200 import indexer_scores, indexer_topk

    q, kk_, w = _inputs(b, tq, tk, h, d, seed=tq * 7 + tk, dtype=dtype)
    qd, kd, wd = q.to(cuda), kk_.to(cuda), w.to(cuda)
    s = indexer_scores(qd, kd, wd)
    ref = oracle.indexer_scores(_np(q), _np(kk_), _np(w))
    scale = np.abs(ref).max() + 1e-6
    assert np.abs(_np(s) - ref).max() <= 2e-6 * scale * max(1, h * d / 64)
    vals, idx = indexer_topk(qd, kd, wd, k)
    kk = min(k, tk)
    assert vals.shape == (b, tq, kk)
    _check_selection_on_own_scores(s, vals, idx, kk)


@pytest.mark.parametrize("offset", [0, 37])
def test_indexer_causal(cuda, offset):
    from linattn_b200 import indexer_scores, indexer_topk

    b, tq, tk, h, d, k = 2, 70, 70 + offset, 4, 64, 16
    q, kk_, w = _inputs(b, tq, tk, h, d, seed=5 + offset)
    qd, kd, wd = q.to(cuda), kk_.to(cuda), w.to(cuda)
    s = indexer_scores(qd, kd, wd, causal=True, offset=offset)
    allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + offset)
    assert np.all(np.isneginf(_np(s)[:, ~allow]))
    vals, idx = indexer_topk(qd, kd, wd, k, causal=True, offset=offset)
    _check_selection_on_own_scores(s, vals, idx, k, causal=True, offset=offset)
    # early queries see fewer than k keys: the padding is (-inf, -1)
    if offset == 0:
        assert idx[0, 0, 0].item() == 0 and torch.all(idx[0, 0, 1:] == -1)
        assert torch.all(torch.isneginf(vals[0, 0, 1:]))
    # the sorted top-k values are those of the float64 oracle's causal top-k
    ov, _ = oracle.indexer_topk(_np(q), _np(kk_), _np(w), k, causal=True, offset=offset)
    assert np.allclose(_np(vals), ov, atol=1e-5)


def test_indexer_chunked_batches(cuda):
    """Several query chunks (small scratch) with B > 1 give the single-chunk result."""
    from linattn_b200 import indexer_topk

    b, tq, tk, h, d, k = 3, 100, 257, 2, 32, 20
    q, kk_, w = _inputs(b, tq, tk, h, d, seed=11)
    qd, kd, wd = q.to(cuda), kk_.to(cuda), w.to(cuda)
    v1, i1 = indexer_topk(qd, kd, wd, k, causal=True, offset=150)
    v2, i2 = indexer_topk(qd, kd, wd, k, causal=True, offset=150, max_scratch_bytes=b * tk * 4 * 9,
                          index_dtype=torch.int32)
    assert i2.dtype == torch.int32
    assert torch.equal(v1, v2) and torch.equal(i1, i2.long())


def test_indexer_fp8_keys_per_64_token_scales(cuda):
    """fp8 e4m3 keys with one fp32 scale per 64 tokens, checked against the oracle on the
    dequantised keys; the codes match the oracle's e4m3 codec."""
    from linattn_b200 import indexer_scores, indexer_topk, quantize_keys_fp8

    b, tq, tk, h, d, k = 1, 96, 1000, 4, 64, 128
    q, kk_, w = _inputs(b, tq, tk, h, d, seed=3, dtype=torch.bfloat16)
    codes, scales = quantize_keys_fp8(kk_.to(cuda), group=64)
    assert scales.shape == (1, 16)
    # codec parity with the oracle
    n = 16 * 64
    xk = np.zeros((b, n, h, d), np.float32)
    xk[:, :tk] = _np(kk_)
    oc, os_ = oracle.quantize_fp8(xk.reshape(b, 16, 64 * h * d), -1)
    assert np.array_equal(codes.view(torch.uint8).cpu().numpy().reshape(b, -1),
                          oc.reshape(b, -1)[:, :tk * h * d])
    assert np.allclose(scales.cpu().numpy(), os_.reshape(b, 16), rtol=0, atol=0)
    qd, wd = q.to(cuda), w.to(cuda)
    s = indexer_scores(qd, codes, wd, k_scale=scales, causal=True, offset=tk - tq)
    kdq = oracle.e4m3_decode(codes.view(torch.uint8).cpu().numpy()).astype(np.float64)
    ref = oracle.indexer_scores(_np(q), kdq, _np(w), k_scale=scales.cpu().numpy(), group=64)
    allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + tk - tq)
    got = _np(s)
    assert np.all(np.isneginf(got[:, ~allow]))
    err = np.abs(got[:, allow] - ref[:, allow]).max()
    assert err <= 1e-5 * (np.abs(ref).max() + 1e-6)
    vals, idx = indexer_topk(qd, codes, wd, k, k_scale=scales, causal=True, offset=tk - tq)
    _check_selection_on_own_scores(s, vals, idx, k, causal=True, offset=tk - tq)


def test_indexer_long_rows_global_path(cuda):
    """Rows longer than the shared-memory stage (32768 keys) and k = 4096."""
    from linattn_b200 import indexer_scores, indexer_topk

    b, tq, tk, h, d, k = 1, 3, 40000, 1, 16, 4096
    q, kk_, w = _inputs(b, tq, tk, h, d, seed=21, w_scale=1.0)
    qd, kd, wd = q.to(cuda), kk_.to(cuda), w.to(cuda)
    s = indexer_scores(qd, kd, wd)
    vals, idx = indexer_topk(qd, kd, wd, k)
    _check_selection_on_own_scores(s, vals, idx, k)


def test_indexer_rejects_bad_arguments(cuda):
    from linattn_b200 import indexer_topk

    q, kk_, w = _inputs(1, 4, 5000, 2, 8, seed=0)
    with pytest.raises(ValueError):
        indexer_topk(q.to(cuda), kk_.to(cuda), w.to(cuda), 4, backend="triton")
    with pytest.raises(ValueError):
        indexer_topk(q.to(cuda), kk_.to(cuda)[:, :, :1], w.to(cuda), 4)
    with pytest.raises(ValueError):
        indexer_topk(q.to(cuda), kk_.to(cuda).to(torch.float8_e4m3fn), w.to(cuda), 4)  # no scales
    with pytest.raises(NotImplementedError):
        indexer_topk(q.to(cuda), kk_.to(cuda), w.to(cuda), 4097)  # k above 4096


@pytest.mark.parametrize("n", [300, 4096, 5000, 16384, 20000, 32768, 40000])
@pytest.mark.parametrize("k", [1, 17, 2048])
def test_row_topk_ties_and_orders(cuda, n, k):
    """Rows with heavy ties (values from a small set): the k-th value's ties go to the
    lowest indices, in value order and in index order, against the oracle."""
    from linattn_b200 import row_topk

    g = torch.Generator().manual_seed(n + k)
    rows = 6
    s = torch.randint(0, 7, (rows, n), generator=g).float() * 0.25 - 0.5
    s[1] = 0.0                                   # one value everywhere
    s[2] = torch.randn(n, generator=g)           # no ties
    s[3, : n // 2] = float("-inf")               # -inf entries
    sd = s.to(cuda)
    kk = min(k, n)
    ref_idx = topk_lowest_index(s.numpy().astype(np.float64), kk)
    ref_val = np.take_along_axis(s.numpy(), ref_idx, -1)
    v, i = row_topk(sd, k)
    assert np.array_equal(i.cpu().numpy(), ref_idx)
    assert np.array_equal(v.cpu().numpy(), ref_val)
    v2, i2 = row_topk(sd, k, sorted=False, index_dtype=torch.int32)
    srt = np.sort(ref_idx, -1)
    assert np.array_equal(i2.cpu().numpy(), srt)
    assert np.array_equal(v2.cpu().numpy(), np.take_along_axis(s.numpy(), srt, -1))


def test_row_topk_causal_index_order(cuda):
    from linattn_b200 import row_topk

    g = torch.Generator().manual_seed(4)
    rows, n, k = 40, 3000, 64
    s = torch.randint(0, 3, (rows, n), generator=g).float()
    v, i = row_topk(s.to(cuda), k, sorted=False, causal=True, first_pos=20)
    for r in range(rows):
        nv = min(n, 20 + r + 1)
        sel = topk_lowest_index(s[r:r + 1, :nv].numpy().astype(np.float64), min(k, nv))[0]
        exp = np.full(k, -1)
        exp[: len(sel)] = np.sort(sel)
        assert np.array_equal(i[r].cpu().numpy(), exp)
        assert torch.all(torch.isneginf(v[r, len(sel):]))


def test_indexer_zero_weights_all_ties(cuda):
    """All scores exactly 0: the first k keys, in both orders (and causal padding)."""
    from linattn_b200 import indexer_topk

    q, kk_, w = _inputs(1, 100, 5000, 4, 64, seed=8, dtype=torch.bfloat16)
    w = torch.zeros_like(w)
    v, i = indexer_topk(q.to(cuda), kk_.to(cuda), w.to(cuda), 300)
    assert torch.equal(i[0].cpu(), torch.arange(300).expand(100, 300))
    v2, i2 = indexer_topk(q.to(cuda), kk_.to(cuda), w.to(cuda), 300, sorted=False, causal=True, offset=250)
    for t in (0, 10, 99):
        nv = min(300, 250 + t + 1)
        assert torch.equal(i2[0, t, :nv].cpu(), torch.arange(nv))
        assert torch.all(i2[0, t, nv:] == -1)


@pytest.mark.parametrize("h,d,kdt", [(2, 128, torch.bfloat16), (8, 32, "fp8"), (1, 64, torch.float16),
                                     (4, 32, torch.bfloat16), (2, 64, "fp8"), (4, 16, torch.bfloat16),
                                     (8, 16, torch.float16), (8, 16, "fp8"), (4, 16, "fp8")])
@pytest.mark.parametrize("tk", [333, 1024])
def test_indexer_tensor_core_shapes(cuda, h, d, kdt, tk):
    """Every tensor-core instantiation class, ragged T_k (odd row stride), B = 2, causal."""
    from linattn_b200 import indexer_scores, indexer_topk, quantize_keys_fp8

    b, tq, k = 2, 70, 40
    qdt = torch.float16 if kdt == torch.float16 else torch.bfloat16
    q, kk_, w = _inputs(b, tq, tk, h, d, seed=h * d + tk, dtype=qdt)
    qd, wd = q.to(cuda), w.to(cuda)
    if kdt == "fp8":
        kd, sc = quantize_keys_fp8(kk_.to(cuda), 64)
        kref = oracle.e4m3_decode(kd.view(torch.uint8).cpu().numpy()).astype(np.float64)
        scn = sc.cpu().numpy()
    else:
        kd, sc = kk_.to(kdt).to(cuda), None
        kref, scn = _np(kd), None
    off = tk - tq
    s = indexer_scores(qd, kd, wd, k_scale=sc, causal=True, offset=off)
    ref = oracle.indexer_scores(_np(q), kref, _np(w), k_scale=scn, group=64)
    allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + off)
    got = _np(s)
    assert np.all(np.isneginf(got[:, ~allow]))
    assert np.abs(got[:, allow] - ref[:, allow]).max() <= 2e-6 * (np.abs(ref).max() + 1e-6) * max(1, h * d / 64)
    vals, idx = indexer_topk(qd, kd, wd, k, k_scale=sc, causal=True, offset=off)
    _check_selection_on_own_scores(s, vals, idx, k, causal=True, offset=off)
    _, idx_u = indexer_topk(qd, kd, wd, k, k_scale=sc, causal=True, offset=off, sorted=False)
    srt = np.sort(np.where(idx.cpu().numpy() < 0, 1 << 40, idx.cpu().numpy()), -1)
    assert np.array_equal(np.where(srt == 1 << 40, -1, srt), idx_u.cpu().numpy())


@pytest.mark.parametrize("n", [1500, 6000])
def test_row_topk_causal_skip_period(cuda, n):
    """Index-order top-k with `skip` leading non-candidates, causal visibility by row
    position modulo `period`, ties among small integers: the warp-per-row path
    (n <= 2048) and the block path (longer rows) against the oracle."""
    from linattn_b200 import row_topk

    g = torch.Generator().manual_seed(n)
    rows, k, skip, period, first_pos = 30, 40, 3, 10, 7
    s = torch.randint(0, 5, (rows, n), generator=g).float()
    v, i = row_topk(s.to(cuda), k, sorted=False, causal=True, first_pos=first_pos, period=period, skip=skip,
                    index_dtype=torch.int32)
    for r in range(rows):
        nv_all = min(n, first_pos + r % period + 1)
        cand = s[r, skip:nv_all].numpy().astype(np.float64)
        exp = np.full(k, -1)
        if cand.size:
            sel = topk_lowest_index(cand[None], min(k, cand.size))[0] + skip
            exp[: sel.size] = np.sort(sel)
        assert np.array_equal(i[r].cpu().numpy(), exp)
