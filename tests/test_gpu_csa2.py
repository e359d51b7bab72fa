"""GPU parity of the CSA2 path: ``csa2_pool_quant`` (pooled + FP4 / FP8 stored KV) bit
for bit against the reference's outputs and the oracle, and the ``cuda_csa2`` plugin
against the reference's chunked / decode outputs (float32, general sparse kernel) and
against the oracle under its own selection (bf16, token-sparse kernel)."""

from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch

from oracle.csa2 import boundary_tied_rows, compressed_kv, csa2_attend, round_to_dtype
from oracle.quest import topk_lowest_index
from tests.conftest import golden

pytestmark = pytest.mark.gpu

TOL_32 = 2e-5
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _np(t):
    return t.detach().float().cpu().numpy()


def _cfg(bits, d=32, **extras):
    from linattn_b200.core import AttnConfig

    return AttnConfig(n_heads=4, n_kv_heads=2, head_dim=d, window_size=24, topk_blocks=3, compress_ratio=8, seed=5,
                      extras={"bits": bits, **extras})


@pytest.mark.parametrize("d", [48, 128])
def test_pool_quant_bit_exact_against_reference(cuda, d):
    from linattn_b200 import csa2_pool_quant

    g = golden("csa2_variant")
    x = torch.from_numpy(g[f"codec_x_d{d}"])
    for name, m, bits in itertools.product(DTYPES, (3, 4), (4, 8, 16)):
        got = csa2_pool_quant(x.to(DTYPES[name]).to(cuda), m, bits)
        assert got.dtype == DTYPES[name] and got.is_contiguous()
        ref = g[f"codec_{name}_d{d}_m{m}_b{bits}"]
        assert np.array_equal(_np(got), ref), (name, m, bits, int((_np(got) != ref).sum()))


@pytest.mark.parametrize("name", ["bf16", "f16"])
@pytest.mark.parametrize("ratio,bits", [(16, 4), (5, 8), (1, 4)])
def test_pool_quant_strided_large_against_oracle(cuda, name, ratio, bits):
    """A (B, T, H, D) cache viewed as (B, H, T, D), ragged tail, D = 128 (4 quant groups)."""
    from linattn_b200 import csa2_pool_quant

    gen = torch.Generator().manual_seed(ratio * 10 + bits)
    b, t, h, d = 2, 4099, 4, 128
    x = (torch.randn(b, t, h, d, generator=gen) * torch.linspace(0.01, 4.0, d)).to(DTYPES[name])
    x[1, 7 * ratio:9 * ratio, 2, 64:96] = 0  # all-zero quantisation groups
    xg = x.to(cuda).transpose(1, 2)
    got = csa2_pool_quant(xg, ratio, bits)
    ref = compressed_kv(x.transpose(1, 2).float().numpy(), ratio, bits, 32, name)
    assert np.array_equal(_np(got), ref), int((_np(got) != ref).sum())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("chunk", [64, 192])
def test_cuda_csa2_variant_golden(cuda, bits, chunk):
    from linattn_b200 import build

    g = golden("csa2_variant")
    var = build("cuda_csa2", _cfg(bits))
    assert np.array_equal(_np(var.q_proj), g[f"q_proj_b{bits}"])
    q, k, v = (torch.from_numpy(g[x]).to(cuda) for x in "qkv")
    out, _ = var.forward(q, k, v, chunk=chunk)
    tied = boundary_tied_rows(g[f"scores_b{bits}"][0], ratio=8, window=24, topk_groups=3, chunk=chunk)
    err = np.abs(_np(out) - g[f"out{chunk}_b{bits}"])[0].max(-1)
    assert err[~tied].max() < TOL_32
    assert tied.mean() < 0.02
    st = var.stats()
    # a tie changes which groups a row reads, never how many
    for key in ("reads_per_query", "groups_per_query", "tokens_equivalent", "bits"):
        assert st[key] == pytest.approx(float(g[f"stats{chunk}_b{bits}_{key}"]), abs=1e-6), key


@pytest.mark.parametrize("bits", [4, 8])
def test_cuda_csa2_variant_decode_golden(cuda, bits):
    from linattn_b200 import build

    g = golden("csa2_variant")
    q, k, v = (torch.from_numpy(g[x]).to(cuda) for x in "qkv")
    var = build("cuda_csa2", _cfg(bits))
    _, st = var.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
    od, _ = var.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
    assert np.abs(_np(od) - g[f"out_decode_b{bits}"]).max() < TOL_32
    assert var.stats()["reads_per_query"] == pytest.approx(float(g[f"reads_decode_b{bits}"]), abs=1e-6)


def _selection_mask(ids, n_groups):
    sel = np.zeros((*ids.shape[:3], n_groups), dtype=bool)
    for idx in np.ndindex(*ids.shape[:3]):
        row = ids[idx]
        sel[idx][row[row >= 0]] = True
    return sel


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bits", [4, 8, 16])
def test_cuda_csa2_token_kernel_path(cuda, d, bits):
    """bf16, head sizes 64 / 128: pooled KV bit-exact with the oracle, the selection the
    exact lowest-index top-k of the eligible groups under the plugin's own scores, and
    the output equal to float64 attention over window + selected groups."""
    from linattn_b200 import build

    gen = torch.Generator().manual_seed(d + bits)
    b, hq, hkv, t, m = 1, 4, 2, 300, 8
    q, k, v = (torch.randn(b, h, t, d, generator=gen).bfloat16() for h in (hq, hkv, hkv))
    cfg = _cfg(bits, d, indexer_heads=4, topk_groups=5, window=40)
    var = build("cuda_csa2", cfg)
    qc, kc_, vc_ = q.to(cuda), k.to(cuda), v.to(cuda)
    out, _ = var.forward(qc, kc_, vc_, chunk=t)
    kc, vc = var.compressed_kv(kc_, vc_)
    assert np.array_equal(_np(kc), compressed_kv(k.float().numpy(), m, bits, 32, "bf16"))
    assert np.array_equal(_np(vc), compressed_kv(v.float().numpy(), m, bits, 32, "bf16"))
    # the selection against the plugin's own fp32 scores
    n_groups = kc.shape[-2]
    ids = var.select_groups(qc, kc, t, 0).cpu().numpy()
    scores = _np(var.indexer_scores(qc, kc)).astype(np.float64)
    pos = np.arange(t)[:, None]
    elig = (np.arange(n_groups)[None, :] + 1) * m <= pos - 40 + 1
    want = topk_lowest_index(np.where(elig, scores, -np.inf), 5)
    want_mask = np.zeros_like(scores, dtype=bool)
    np.put_along_axis(want_mask, want, True, axis=-1)
    assert np.array_equal(_selection_mask(ids, n_groups), want_mask & elig)
    # the output: float64 attention over [window tokens, selected pooled rows]
    win_mask = (np.arange(t)[None, :] <= pos) & (pos - np.arange(t)[None, :] < 40)
    allow = np.concatenate([np.broadcast_to(win_mask, (b, hq, t, t)), want_mask & elig], axis=-1)
    k_all = np.concatenate([k.float().numpy(), _np(kc)], axis=2).astype(np.float64)
    v_all = np.concatenate([v.float().numpy(), _np(vc)], axis=2).astype(np.float64)
    kr, vr = np.repeat(k_all, 2, axis=1), np.repeat(v_all, 2, axis=1)
    s = np.einsum("bhtd,bhsd->bhts", q.float().numpy().astype(np.float64), kr) / np.sqrt(d)
    s = np.where(allow, s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    ref = np.einsum("bhts,bhsd->bhtd", p / p.sum(-1, keepdims=True), vr)
    err = np.abs(_np(out) - ref)
    assert np.all(err <= 2e-3 + 2.0 ** -8 * np.abs(ref)), err.max()
    st = var.stats()
    assert st["groups_per_query"] == pytest.approx((want_mask & elig).sum(-1).mean(), rel=1e-9)
    assert st["reads_per_query"] == pytest.approx(allow.sum(-1).mean(), rel=1e-9)


@pytest.mark.parametrize("t", [1, 5, 30])
def test_cuda_csa2_short_sequences(cuda, t):
    """No complete group before the window (window only), a single partial group."""
    from linattn_b200 import build

    gen = torch.Generator().manual_seed(t)
    q, k, v = (torch.randn(1, h, t, 32, generator=gen) for h in (4, 2, 2))
    var = build("cuda_csa2", _cfg(4))
    out, _ = var.forward(q.to(cuda), k.to(cuda), v.to(cuda), chunk=t)
    ref, stats = csa2_attend(q.numpy(), k.numpy(), v.numpy(), _np(var.q_proj), np.full(4, 0.25, np.float32),
                             ratio=8, bits=4, group=32, window=24, topk_groups=3)
    assert np.abs(_np(out) - ref).max() < TOL_32
    assert var.stats()["reads_per_query"] == pytest.approx(stats["reads_per_query"], rel=1e-9)


def test_pool_quant_rejects_bad_arguments(cuda):
    from linattn_b200 import csa2_pool_quant

    x = torch.randn(1, 1, 16, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        csa2_pool_quant(x, 4, bits=5)
    with pytest.raises(Exception, match="groups of 32"):
        csa2_pool_quant(x, 4, bits=4, group=16)
    with pytest.raises(Exception, match="D <= 256"):
        csa2_pool_quant(torch.randn(1, 1, 16, 320, device=cuda, dtype=torch.bfloat16), 4)
    assert round_to_dtype(np.float32([1.0]), "bf16")[0] == 1.0


@pytest.mark.parametrize("name", ["bf16", "f32"])
@pytest.mark.parametrize("bits", [4, 8])
def test_pool_quant_vector_and_scalar_forms(cuda, name, bits):
    """D = 96 (12 threads per pooled row: a CTA's last threads idle) on the vector form,
    and the same values through a view one element off 16-byte alignment (the scalar
    form): both bit-exact with the oracle."""
    from linattn_b200 import csa2_pool_quant

    gen = torch.Generator().manual_seed(bits + len(name))
    b, h, t, d, ratio = 2, 3, 1001, 96, 7
    x = (torch.randn(b, h, t, d + 1, generator=gen) * torch.linspace(0.02, 3.0, d + 1)).to(DTYPES[name])
    ref = compressed_kv(x[..., 1:].float().numpy(), ratio, bits, 32, name)
    xg = x.to(cuda)
    aligned = csa2_pool_quant(xg[..., 1:].contiguous(), ratio, bits)
    shifted = csa2_pool_quant(xg[..., 1:], ratio, bits)  # base one element past alignment
    assert np.array_equal(_np(aligned), ref)
    assert np.array_equal(_np(shifted), ref)
