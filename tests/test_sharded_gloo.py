"""Host side of the sequence-sharded decode on two CPU ranks (gloo): page ranges, the
rank-major layout of the exchanges, and that the global top-k of the gathered
candidates (score desc, lowest page on ties) equals the top-k over the whole cache."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _merge_reference(all_s: np.ndarray, all_i: np.ndarray, topk: int) -> np.ndarray:
    """Global top-k of rank-major candidates by (score desc, page asc)."""
    r, b, h, k = all_s.shape
    s = np.transpose(all_s, (1, 2, 0, 3)).reshape(b, h, r * k)
    i = np.transpose(all_i, (1, 2, 0, 3)).reshape(b, h, r * k)
    out = np.full((b, h, topk), -1, np.int64)
    for bi in range(b):
        for hi in range(h):
            ok = i[bi, hi] >= 0
            order = np.lexsort((i[bi, hi][ok], -s[bi, hi][ok]))[:topk]
            out[bi, hi, : len(order)] = i[bi, hi][ok][order]
    return out


def _worker(rank, world, port, seed, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from linattn_b200.sharded import exchange_candidates, exchange_packed, exchange_partials, shard_page_ranges

        rng = np.random.default_rng(seed)
        b, h, n_pages, topk = 2, 4, 37, 6
        # the whole cache's page scores (quantised so that ties occur), same on every rank
        scores = np.round(rng.standard_normal((b, h, n_pages)) * 4) / 4
        lo, hi = shard_page_ranges(n_pages, world, rank)
        local = scores[:, :, lo:hi]
        kk = min(topk, hi - lo)
        li = oracle.topk_lowest_index(local, kk)
        ls = np.take_along_axis(local, li, -1)
        pad = topk - kk
        ids = np.concatenate([li + lo, np.full((b, h, pad), -1)], -1).astype(np.int32)
        sc = np.concatenate([ls, np.full((b, h, pad), -np.inf)], -1).astype(np.float32)
        all_s, all_i = exchange_candidates(torch.from_numpy(sc), torch.from_numpy(ids))
        assert tuple(all_s.shape) == (world, b, h, topk)
        assert np.array_equal(all_i[rank].numpy(), ids)  # rank-major
        merged = _merge_reference(all_s.numpy(), all_i.numpy(), topk)
        want = oracle.topk_lowest_index(scores, topk)
        assert np.array_equal(merged, want)
        o = torch.full((3, 5), float(rank))
        lse = torch.full((3,), float(rank))
        all_o, all_l = exchange_partials(o, lse)
        assert torch.equal(all_o[1], torch.ones(3, 5)) and torch.equal(all_l[0], torch.zeros(3))
        # packed buffers: one (2, B, H, K) int32 candidate block per rank, rank-major
        cand = torch.stack([torch.from_numpy(sc).view(torch.int32), torch.from_numpy(ids)])
        allc = exchange_packed(cand)
        assert tuple(allc.shape) == (world, 2, b, h, topk)
        assert torch.equal(allc[:, 0].view(torch.float32), all_s) and torch.equal(allc[:, 1], all_i)
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("seed", [0, 1])
def test_sharded_exchange_and_merge_two_ranks(seed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, seed, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(0, "ok"), (1, "ok")], results


def test_shard_page_ranges_partition():
    from linattn_b200.sharded import shard_page_ranges

    for n in (1, 7, 16384):
        for world in (1, 2, 3, 8):
            ranges = [shard_page_ranges(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1
