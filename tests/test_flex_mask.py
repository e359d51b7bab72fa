"""Block-mask coverage utilities (``linattn_b200.flex_mask``; the reference's
``kernels/flex_mask.py:35-72`` names): the reduction of a token mask is a superset
of it and equals the dense any-reduction, a dropped block is caught, the oracle's
block lists (configuration-4 windows, MoBA per-token routing) cover the token masks
they stand for, and the FlexAttention ``BlockMask`` built from lists holds the same
cells.  CPU only."""
import numpy as np
import torch

from oracle.blocks import block_mask_to_token_mask, moba_select, window_block_select
from linattn_b200.flex_mask import (check_block_mask, check_lists_cover, flex_available, lists_to_block_mask,
                                   mask_to_block_mask, to_block_mask)


def test_reduction_is_superset_and_drop_is_caught():
    gen = torch.Generator().manual_seed(0)
    mask = torch.rand(2, 3, 150, 200, generator=gen) < 0.02
    reduced = mask_to_block_mask(mask, 64, 32)
    assert reduced.shape == (2, 3, 3, 7)
    ok, coverage = check_block_mask(mask, reduced, 64, 32)
    assert ok and 0.0 < coverage <= 1.0
    # drop one kept block that holds a read token: the check must fail
    bb, hh, qb, kb = [int(x) for x in reduced.nonzero()[0]]
    broken = reduced.clone()
    broken[bb, hh, qb, kb] = False
    assert not check_block_mask(mask, broken, 64, 32)[0]
    # the same cells as a dense any-reduction over padded 64 x 32 tiles
    pad = torch.zeros(2, 3, 192, 224, dtype=torch.bool)
    pad[..., :150, :200] = mask
    assert torch.equal(reduced, pad.view(2, 3, 3, 64, 7, 32).any(3).any(-1))


def test_flex_block_mask_from_lists():
    if not flex_available():
        return
    gen = torch.Generator().manual_seed(3)
    mask = torch.rand(1, 2, 256, 256, generator=gen) < 0.01
    reduced = mask_to_block_mask(mask, 64, 64)
    bm = to_block_mask(mask, 64, 64)
    assert torch.equal(bm.to_dense().bool(), reduced)


def test_window_lists_cover_their_token_mask():
    rng = np.random.default_rng(1)
    b, hq, hkv, t, d, block = 1, 4, 2, 1024, 32, 64
    q = rng.standard_normal((b, hq, t, d)).astype(np.float32)
    k = rng.standard_normal((b, hkv, t, d)).astype(np.float32)
    ids, counts = window_block_select(q, k, block, 3, window_blocks=2, sink_blocks=1)
    n_kb = t // block
    ids_t, counts_t = torch.from_numpy(ids), torch.from_numpy(counts)
    sel = lists_to_block_mask(ids_t, n_kb, counts_t)
    # the token mask the lists stand for, with causality: exactly covered
    causal = np.tril(np.ones((t, t), dtype=bool))
    tok = block_mask_to_token_mask(sel.numpy(), block, block, t, t) & causal
    ok, coverage = check_lists_cover(torch.from_numpy(tok), ids_t, block, counts_t, rows_per_list=block)
    assert ok
    assert abs(coverage - sel.float().mean().item()) < 1e-12
    # a list missing one of its blocks no longer covers the mask
    cut = counts_t.clone()
    cut[0, 0, -1] -= 1
    assert not check_lists_cover(torch.from_numpy(tok), ids_t, block, cut, rows_per_list=block)[0]


def test_moba_per_token_routing_covers_oracle_mask():
    rng = np.random.default_rng(2)
    b, hq, hkv, t, d, block, topk = 1, 2, 1, 256, 16, 32, 2
    q = rng.standard_normal((b, hq, t, d)).astype(np.float32)
    k = rng.standard_normal((b, hkv, t, d)).astype(np.float32)
    mask = moba_select(q, k, block, topk)  # (B, H, T, T) token mask of the routing
    # per-token lists from the mask itself (ascending, -1 padded)
    sel = mask.reshape(b, hq, t, t // block, block).any(-1)
    n = int(sel.sum(-1).max())
    ids = np.full((b, hq, t, n), -1, dtype=np.int32)
    for bi in range(b):
        for h in range(hq):
            for ti in range(t):
                row = np.nonzero(sel[bi, h, ti])[0]
                ids[bi, h, ti, : row.size] = row
    ok, _ = check_lists_cover(torch.from_numpy(mask), torch.from_numpy(ids), block, rows_per_list=1)
    assert ok
    assert np.array_equal(lists_to_block_mask(torch.from_numpy(ids), t // block).numpy(), sel)
