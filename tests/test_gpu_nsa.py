"""GPU parity of the ``cuda_nsa`` plugin: the three branches, the chunked / decode
outputs and the fitted gates against the reference's outputs (float32, general sparse
kernel), and the bf16 token-sparse / tcgen05 prefill paths against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import dense_attention
from oracle.nsa import nsa_block_scores, nsa_branches, nsa_fill_rows, nsa_select
from tests.conftest import golden

pytestmark = pytest.mark.gpu

TOL_32 = 2e-5


def _np(t):
    return t.detach().float().cpu().numpy()


def _cfg(selected=3, **kw):
    from linattn_b200.core import AttnConfig

    base = dict(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=24, topk_blocks=selected,
                compress_ratio=8, seed=5)
    base.update(kw)
    return AttnConfig(**base)


def _defined_rows(g, selected=3):
    sc = g["block_scores"][0]
    h, t, n_kb = sc.shape
    ok = np.ones((h, t), dtype=bool)
    ok[:, nsa_fill_rows(t, 16, selected, n_kb)] = False
    for hh in range(h):
        for tt in range(t):
            s = np.sort(sc[hh, tt][np.arange(n_kb) * 16 <= tt])[::-1]
            if s.size > selected and abs(s[selected - 1] - s[selected]) <= 1e-6 * max(1.0, abs(s[selected])):
                ok[hh, tt] = False
    return ok


def _qkv(g, cuda):
    return (torch.from_numpy(g[x]).to(cuda) for x in "qkv")


def test_cuda_nsa_branches_golden(cuda):
    from linattn_b200 import build

    g = golden("nsa_variant")
    q, k, v = _qkv(g, cuda)
    var = build("cuda_nsa", _cfg())
    ok = _defined_rows(g)
    assert np.abs(_np(var.branch_compression(q, k, v, 0)) - g["o_cmp"]).max() < TOL_32
    assert np.abs(_np(var.branch_window(q, k, v, 0)) - g["o_win"]).max() < TOL_32
    err = np.abs(_np(var.branch_selection(q, k, v, 0)) - g["o_slc"])[0].max(-1)
    assert err[ok].max() < TOL_32
    # the selected blocks, as a token mask, on the rows the reference defines
    ids, counts = var.selection_lists(q, k, 0)
    ids, counts = ids.cpu().numpy()[0], counts.cpu().numpy()[0]
    sel = np.zeros((4, 192, 12), dtype=bool)
    for hh in range(4):
        for tt in range(192):
            sel[hh, tt, ids[hh, tt, :counts[hh, tt]]] = True
    tok = np.repeat(sel, 16, axis=-1)
    assert np.array_equal(tok[ok], g["sel_mask"][0][ok])


@pytest.mark.parametrize("chunk", [64, 192])
def test_cuda_nsa_variant_golden(cuda, chunk):
    from linattn_b200 import build

    g = golden("nsa_variant")
    q, k, v = _qkv(g, cuda)
    var = build("cuda_nsa", _cfg())
    out, _ = var.forward(q, k, v, chunk=chunk)
    ok = _defined_rows(g)
    assert np.abs(_np(out) - g[f"out{chunk}"])[0].max(-1)[ok].max() < TOL_32
    st = var.stats()
    assert st["reads_per_query"] == pytest.approx(float(g[f"stats{chunk}_reads_per_query"]))
    if chunk == 64:
        assert st["selected_blocks_per_query"] == pytest.approx(float(g["stats64_selected_blocks_per_query"]),
                                                                rel=1e-6)


def test_cuda_nsa_single_block_and_decode_golden(cuda):
    from linattn_b200 import build

    g = golden("nsa_variant")
    q, k, v = _qkv(g, cuda)
    var = build("cuda_nsa", _cfg(selected=1))
    out, _ = var.forward(q, k, v, chunk=192)
    assert np.abs(_np(out) - g["out192_k1"]).max() < TOL_32
    assert var.stats()["selected_blocks_per_query"] == pytest.approx(
        float(g["stats192_k1_selected_blocks_per_query"]), rel=1e-6)
    var = build("cuda_nsa", _cfg())
    _, st = var.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
    od, _ = var.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
    assert np.abs(_np(od) - g["out_decode"]).max() < TOL_32


def test_cuda_nsa_fit_gates_golden(cuda):
    from linattn_b200 import build

    g = golden("nsa_variant")
    q, k, v = _qkv(g, cuda)
    var = build("cuda_nsa", _cfg(selected=1))
    loss = var.fit_gates(q, k, v, steps=25, lr=0.05)
    assert loss == pytest.approx(float(g["fit_loss"]), rel=1e-4)
    assert np.abs(_np(var.gates) - g["gates_fit"]).max() < 1e-4
    assert var.gate_mode == "learned"
    out, _ = var.forward(q, k, v, chunk=192)
    assert np.abs(_np(out) - g["out_learned"]).max() < 1e-4


@pytest.mark.parametrize("d,block,selected", [(128, 64, 2), (64, 16, 3)])
def test_cuda_nsa_bf16_paths(cuda, d, block, selected):
    """bf16: the compression branch on the tcgen05 prefill with its pooled causal rule
    (D = 128) or the token-sparse kernel (D = 64), the window branch on the token-sparse
    kernel, selection on the tcgen05 prefill (64-token blocks, D = 128) or the general
    kernel; each branch
    against float64 attention (pooled rows rounded to bf16 as the reference pools), the
    lists bit-exact against the oracle's selection on the kernel's own fp32 scores."""
    from linattn_b200 import build

    gen = torch.Generator().manual_seed(d + block)
    b, hq, hkv, t = 1, 4, 2, 300
    q, k, v = (torch.randn(b, h, t, d, generator=gen).bfloat16() for h in (hq, hkv, hkv))
    cfg = _cfg(selected, head_dim=d, block_size=block, window_size=40)
    var = build("cuda_nsa", cfg)
    qc, kc, vc = q.to(cuda), k.to(cuda), v.to(cuda)
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    o_cmp, o_slc_oracle, o_win, sel_oracle = nsa_branches(qn, kn, vn, compress=8, block=block, selected=selected,
                                                          window=40, dtype="bf16")
    tol = 2e-3 + 2.0 ** -8 * np.abs(o_cmp)
    assert np.all(np.abs(_np(var.branch_compression(qc, kc, vc, 0)) - o_cmp) <= tol)
    assert np.all(np.abs(_np(var.branch_window(qc, kc, vc, 0)) - o_win) <= 2e-3 + 2.0 ** -8 * np.abs(o_win))
    # selection: the plugin's lists bit-exact against the oracle's selection rule applied
    # to the kernel's own fp32 scores (recorded by the same kernel through scores_out)
    from linattn_b200.blocks import block_score_topk
    from linattn_b200.csa2 import csa2_pool_quant

    ids, counts = var.selection_lists(qc, kc, 0)
    ids, counts = ids.cpu().numpy(), counts.cpu().numpy()
    n_kb = -(-t // block)
    sel = np.zeros((b, hq, t, n_kb), dtype=bool)
    for idx in np.ndindex(b, hq, t):
        sel[idx][ids[idx][:counts[idx]]] = True
    own_sc = torch.full((b, hq, t, n_kb), float("-inf"), device=cuda)
    block_score_topk(qc, csa2_pool_quant(kc, block, 16), selected, scale=d ** -0.5, first_pos=0, key_block=block,
                     merge_pos=0, own_div=block, scores_out=own_sc)
    want = nsa_select(own_sc.cpu().numpy().astype(np.float64), block, selected)
    assert np.array_equal(sel, want)
    # and those scores against float64 on the bf16-pooled keys
    sc = nsa_block_scores(qn, kn, block, "bf16")
    fin = np.isfinite(own_sc.cpu().numpy())
    assert np.allclose(own_sc.cpu().numpy()[fin], sc[fin], rtol=1e-5, atol=1e-5)
    # rows where float64 and the kernel's fp32 scores would rank differently are rare
    assert (np.array_equal(sel, sel_oracle) or (sel != sel_oracle).any(-1).mean() < 0.01)
    # the selection branch against float64 attention over the plugin's own blocks
    tok = np.repeat(sel, block, axis=-1)[..., :t]
    ref = dense_attention(qn, kn, vn, causal=False, mask=tok)
    got = _np(var.branch_selection(qc, kc, vc, 0))
    assert np.all(np.abs(got - ref) <= 2e-3 + 2.0 ** -8 * np.abs(ref))
    # the combination: uniform gates over the three branch outputs
    out, _ = var.forward(qc, kc, vc, chunk=t)
    mixed = (o_cmp + ref + o_win) / 3.0
    assert np.all(np.abs(_np(out) - mixed) <= 4e-3 + 2.0 ** -8 * np.abs(mixed))
    del o_slc_oracle


@pytest.mark.parametrize("offset,t", [(37, 150), (200, 130)])
def test_cuda_nsa_window_and_compression_at_offset(cuda, offset, t):
    """The plugin's tensor-core window and compression branches for queries that start
    mid-sequence (an offset that is not a multiple of 64, so the per-64-query block
    ranges straddle key blocks), against float64 attention over the oracle's read sets."""
    from linattn_b200 import build

    gen = torch.Generator().manual_seed(offset + t)
    b, hq, hkv, d = 1, 4, 2, 128
    tk = offset + t
    q = torch.randn(b, hq, t, d, generator=gen).bfloat16()
    k, v = (torch.randn(b, hkv, tk, d, generator=gen).bfloat16() for _ in range(2))
    var = build("cuda_nsa", _cfg(2, head_dim=d, block_size=64, window_size=40))
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    o_cmp, _, o_win, _ = nsa_branches(qn, kn, vn, compress=8, block=64, selected=2, window=40, offset=offset,
                                      dtype="bf16")
    qc, kc, vc = q.to(cuda), k.to(cuda), v.to(cuda)
    got_w = _np(var.branch_window(qc, kc, vc, offset))
    got_c = _np(var.branch_compression(qc, kc, vc, offset))
    assert np.all(np.abs(got_w - o_win) <= 2e-3 + 2.0 ** -8 * np.abs(o_win)), np.abs(got_w - o_win).max()
    assert np.all(np.abs(got_c - o_cmp) <= 2e-3 + 2.0 ** -8 * np.abs(o_cmp)), np.abs(got_c - o_cmp).max()


@pytest.mark.parametrize("c,offset", [(3, 5), (16, 0), (1, 7), (3, -2), (8, -5)])
def test_prefill_pooled_causal_rule(cuda, c, offset):
    """``block_sparse_prefill(causal=c)``: key j read by the query at p iff
    j * c <= p + c - 1 (c = 1: the usual causal rule), with a partial last block; a
    negative offset puts the first rows at -c < p < 0, where key 0 is already read."""
    from linattn_b200.blocks import block_sparse_prefill

    gen = torch.Generator().manual_seed(c + offset)
    b, hq, hkv, tq, tk, d = 1, 4, 2, 200, 100, 128
    q = torch.randn(b, hq, tq, d, generator=gen).bfloat16()
    k, v = (torch.randn(b, hkv, tk, d, generator=gen).bfloat16() for _ in range(2))
    n_blk = -(-tk // 64)
    ids = torch.arange(n_blk, dtype=torch.int32).view(1, 1, 1, n_blk).expand(b, hq, 1, n_blk)
    out = block_sparse_prefill(q.to(cuda), k.to(cuda), v.to(cuda), ids.to(cuda), rows_per_list=tq, causal=c,
                               offset=offset)
    pos = (np.arange(tq) + offset)[:, None]
    allow = np.broadcast_to(np.arange(tk)[None, :] * c <= pos + c - 1, (b, hq, tq, tk))
    ref = dense_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False, mask=allow)
    assert np.all(np.abs(_np(out) - ref) <= 2e-3 + 2.0 ** -8 * np.abs(ref)), np.abs(_np(out) - ref).max()


@pytest.mark.parametrize("w,offset,tq", [(40, 7, 200), (100, 0, 257), (1, 3, 70)])
def test_prefill_window_rule(cuda, w, offset, tq):
    """``block_sparse_prefill(window=w)``: the query at p reads keys [p - w + 1, p] of its
    listed blocks (the NSA window branch's read set), per-64-row block lists."""
    from linattn_b200.blocks import block_sparse_prefill

    gen = torch.Generator().manual_seed(w + offset)
    b, hq, hkv, d = 1, 4, 2, 128
    tk = offset + tq
    q = torch.randn(b, hq, tq, d, generator=gen).bfloat16()
    k, v = (torch.randn(b, hkv, tk, d, generator=gen).bfloat16() for _ in range(2))
    n_kb, n_qb = -(-tk // 64), -(-tq // 64)
    ids = torch.arange(n_kb, dtype=torch.int32).view(1, 1, 1, n_kb).expand(b, hq, n_qb, n_kb)  # every block
    out = block_sparse_prefill(q.to(cuda), k.to(cuda), v.to(cuda), ids.contiguous().to(cuda), rows_per_list=64,
                               causal=True, window=w, offset=offset)
    pos = (np.arange(tq) + offset)[:, None]
    kj = np.arange(tk)[None, :]
    allow = np.broadcast_to((kj <= pos) & (pos - kj < w), (b, hq, tq, tk))
    ref = dense_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False, mask=allow)
    assert np.all(np.abs(_np(out) - ref) <= 2e-3 + 2.0 ** -8 * np.abs(ref)), np.abs(_np(out) - ref).max()
