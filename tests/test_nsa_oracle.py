"""The NSA oracle (``oracle/nsa.py``) pinned to the reference's own outputs
(``tests/golden/nsa_variant.npz``, written by ``make_golden.py`` from ``NSAAttention``):
the three branches, the selection mask, the chunked / decode outputs on every row whose
selection the reference defines, the full forward and the fitted gates with one selected
block, and the accounting of the ``cuda_nsa`` plugin.  CPU only."""

import numpy as np
import pytest
import torch

from oracle.attention import dense_attention
from oracle.nsa import nsa_attend, nsa_branches, nsa_fill_rows, nsa_forward
from tests.conftest import golden

KW = dict(compress=8, block=16, selected=3, window=24)


def _defined_rows(g, selected=3):
    """(H, T): rows the reference defines (no fill from later blocks, no exact tie at the
    boundary of the block top-k)."""
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


def test_branches_and_selection_against_reference():
    g = golden("nsa_variant")
    o_cmp, o_slc, o_win, sel = nsa_branches(g["q"], g["k"], g["v"], **KW)
    ok = _defined_rows(g)
    assert ok.mean() > 0.8
    assert np.abs(o_cmp - g["o_cmp"]).max() < 2e-5
    assert np.abs(o_win - g["o_win"]).max() < 2e-5
    assert np.abs(o_slc - g["o_slc"])[0].max(-1)[ok].max() < 2e-5
    tok = np.repeat(sel, 16, axis=-1)[..., :192][0]
    assert np.array_equal(tok[ok], g["sel_mask"][0][ok])


@pytest.mark.parametrize("chunk", [64, 192])
def test_forward_against_reference(chunk):
    g = golden("nsa_variant")
    out, stats = nsa_forward(g["q"], g["k"], g["v"], chunk=chunk, **KW)
    ok = _defined_rows(g)
    assert np.abs(out - g[f"out{chunk}"])[0].max(-1)[ok].max() < 2e-5
    if chunk == 64:  # the last chunk (positions 128..191) has no fill rows
        assert stats["selected_blocks_per_query"] == pytest.approx(float(g["stats64_selected_blocks_per_query"]))


def test_decode_and_single_block_against_reference():
    g = golden("nsa_variant")
    q, k, v = g["q"], g["k"], g["v"]
    out, _ = nsa_attend(q[:, :, 191:], k, v, offset=191, **KW)
    assert np.abs(out - g["out_decode"]).max() < 2e-5
    kw1 = dict(KW, selected=1)
    out, stats = nsa_forward(q, k, v, chunk=192, **kw1)
    assert np.abs(out - g["out192_k1"]).max() < 2e-5
    assert stats["selected_blocks_per_query"] == pytest.approx(float(g["stats192_k1_selected_blocks_per_query"]))


def test_fitted_gates_against_reference():
    """Adam on the gates over the oracle's branch outputs reproduces the reference's
    ``fit_gates`` (the branches do not depend on the gates)."""
    g = golden("nsa_variant")
    q, k, v = g["q"], g["k"], g["v"]
    branches = [torch.from_numpy(x).float() for x in nsa_branches(q, k, v, **dict(KW, selected=1))[:3]]
    target = torch.from_numpy(dense_attention(q, k, v, causal=True)).float()
    gates = torch.nn.Parameter(torch.from_numpy(g["gates_init"]).clone())
    opt = torch.optim.Adam([gates], lr=0.05)
    for _ in range(25):
        opt.zero_grad()
        w = torch.sigmoid(gates)
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-9)
        out = sum(w[:, i].view(1, -1, 1, 1) * branches[i] for i in range(3))
        loss = torch.nn.functional.mse_loss(out, target)
        loss.backward()
        opt.step()
    assert float(loss.detach()) == pytest.approx(float(g["fit_loss"]), rel=1e-5)
    assert np.abs(gates.detach().numpy() - g["gates_fit"]).max() < 1e-5
    out, _ = nsa_attend(q, k, v, gates=gates.detach().numpy(), **dict(KW, selected=1))
    assert np.abs(out - g["out_learned"]).max() < 2e-5


def test_plugin_parameters_and_accounting():
    from linattn_b200.core import AttnConfig
    from linattn_b200.registry import build

    g = golden("nsa_variant")
    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=24, topk_blocks=3,
                     compress_ratio=8, seed=5)
    assert np.array_equal(build("cuda_nsa", cfg).gates.detach().numpy(), g["gates_init"])
    rows = iter(g["accounting"])
    for extras in ({}, {"compress_ratio": 4, "selected_blocks": 6}):
        var = build("cuda_nsa", AttnConfig(n_heads=8, n_kv_heads=2, head_dim=64, extras=dict(extras)))
        for n in (5, 100, 4096):
            got = [var.read_budget(n), var.memory_bytes(n), var.flops(n), var.read_budget(n, 3),
                   var.memory_bytes(n, 3), var.flops(n, 3)]
            assert np.array_equal(np.array(got, np.float64), next(rows)), (extras, n)
    assert build("cuda_nsa", cfg).stats()["reads_per_query"] == 24 + 3 * 16
