"""The CSA2 oracle (``oracle/csa2.py``) pinned to the reference's own outputs
(``tests/golden/csa2_variant.npz``, written by ``make_golden.py`` from
``CSA2Attention``): the pooled + quantised KV bit for bit in bf16 / f16 / f32, the
chunked and decode outputs and stats in float32, and the accounting formulas of the
``cuda_csa2`` plugin.  CPU only."""

import itertools

import numpy as np
import pytest

from oracle.csa2 import (FP4_GRID, boundary_tied_rows, compressed_kv, csa2_attend, csa2_forward, quant_roundtrip,
                         round_to_dtype)
from tests.conftest import golden

CFG = dict(ratio=8, group=32, window=24, topk_groups=3)
W = np.full(4, 0.25, np.float32)


@pytest.mark.parametrize("d", [48, 128])
def test_codec_bit_exact_against_reference(d):
    g = golden("csa2_variant")
    x = g[f"codec_x_d{d}"]
    for dt, m, bits in itertools.product(("bf16", "f16", "f32"), (3, 4), (4, 8, 16)):
        ref = g[f"codec_{dt}_d{d}_m{m}_b{bits}"]
        got = compressed_kv(round_to_dtype(x, dt), m, bits, 32, dt)
        assert got.shape == ref.shape
        assert np.array_equal(got, ref), (dt, m, bits, int((got != ref).sum()))


def test_fp4_rounding_rules():
    # a group whose absmax maps to 6: the other entries land on exact grid midpoints
    # (ties keep the smaller magnitude, argmin's first index), signs are kept and -0
    # stays a zero
    x = np.zeros(32, np.float32)
    x[:8] = [6.0, 0.25, -0.75, 1.25, 1.75, 2.5, -3.5, 5.0]
    x_hat, codes, scales = quant_roundtrip(x, 4)
    assert scales[0] == np.float32(1.0)
    assert list(x_hat[:8]) == [6.0, 0.0, -0.5, 1.0, 1.5, 2.0, -3.0, 4.0]
    assert list(codes[:8]) == [7, 0, 9, 2, 3, 4, 13, 6]
    assert set(np.unique(np.abs(x_hat))) <= set(FP4_GRID.tolist())
    # an all-zero group takes the 1e-8 clamp and stays zero
    z_hat, _, z_scale = quant_roundtrip(np.zeros(32, np.float32), 4)
    assert np.all(z_hat == 0) and z_scale[0] == np.float32(1e-8) / np.float32(6.0)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("chunk", [64, 192])
def test_variant_against_reference(bits, chunk):
    g = golden("csa2_variant")
    out, stats = csa2_forward(g["q"], g["k"], g["v"], g[f"q_proj_b{bits}"], W, chunk=chunk, bits=bits, **CFG)
    tied = boundary_tied_rows(g[f"scores_b{bits}"][0], ratio=8, window=24, topk_groups=3, chunk=chunk)
    err = np.abs(out - g[f"out{chunk}_b{bits}"])[0].max(-1)
    assert tied.mean() < 0.02
    assert err[~tied].max() < 2e-5
    for key in ("reads_per_query", "groups_per_query", "tokens_equivalent", "bits"):
        assert stats[key] == pytest.approx(float(g[f"stats{chunk}_b{bits}_{key}"]), abs=1e-9)


@pytest.mark.parametrize("bits", [4, 8])
def test_decode_against_reference(bits):
    g = golden("csa2_variant")
    q, k, v = g["q"], g["k"], g["v"]
    out, stats = csa2_attend(q[:, :, 191:], k, v, g[f"q_proj_b{bits}"], W, offset=191, bits=bits, **CFG)
    assert np.abs(out - g[f"out_decode_b{bits}"]).max() < 2e-5
    assert stats["reads_per_query"] == pytest.approx(float(g[f"reads_decode_b{bits}"]), abs=1e-9)


def test_plugin_accounting_matches_reference():
    from linattn_b200.core import AttnConfig
    from linattn_b200.registry import build

    acct = golden("csa2_variant")["accounting"]
    rows = iter(acct)
    for extras in ({}, {"bits": 8, "cross_layer_group": 2}, {"bits": 16, "compress_ratio": 4, "topk_groups": 9}):
        var = build("cuda_csa2", AttnConfig(n_heads=8, n_kv_heads=2, head_dim=64, extras=dict(extras)))
        for n in (5, 100, 4096):
            want = next(rows)
            got = [var.read_budget(n), var.memory_bytes(n), var.selection_flops(n), var.read_budget(n, 3),
                   var.memory_bytes(n, 3)]
            assert np.array_equal(np.array(got, np.float64), want), (extras, n, got, want)
