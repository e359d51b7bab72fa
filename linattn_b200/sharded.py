"""Sequence-sharded Quest decode across GPUs (the million-token configuration).

Every rank holds a contiguous slice of each sequence's KV pages (``PagedKVCache`` of
the slice, pages ``[page_lo_b, page_hi_b)`` of sequence ``b``).  One decode step:

1. local selection (the fused Quest kernel) gives each query head its top-K local pages
   and their scores; only the rank holding a sequence's last page forces it in, only
   the rank holding page 0 forces the sink pages;
2. the (score, global page) candidates are all-gathered (rank-major);
3. every rank takes the same global top-K per head (``linattn_shard_merge``: score
   desc, lowest page on ties, as the single-cache selection) and keeps the GQA union
   of the selected pages it owns;
4. attention over those pages gives fp32 partial ``(o, lse)`` (``lse = -inf`` for a rank
   that owns none of them);
5. the partials are all-gathered and merged by the log-sum-exp combine kernel.

The two exchanges (``exchange_candidates``, ``exchange_partials``) are plain
``torch.distributed.all_gather_into_tensor`` calls on the process group (NCCL over
NVLink between GPUs; any backend for testing the layout on CPU).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from linattn_b200 import _lib as L
from linattn_b200.paged import PagedKVCache, QuestDecoder

__all__ = ["ShardedQuestDecoder", "exchange_candidates", "exchange_partials", "shard_page_ranges"]


def shard_page_ranges(n_pages: int, world: int, rank: int) -> Tuple[int, int]:
    """Pages ``[lo, hi)`` of a sequence of ``n_pages`` pages held by ``rank`` (contiguous,
    as equal as possible, earlier ranks first)."""
    base, extra = divmod(n_pages, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def exchange_candidates(scores: torch.Tensor, ids: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather ``(B, H_q, K)`` candidate scores / global ids into ``(R, B, H_q, K)``."""
    world = dist.get_world_size(group)
    # concatenated along dim 0 (the form every backend accepts), viewed rank-major
    out_s = scores.new_empty((world * scores.shape[0], *scores.shape[1:]))
    out_i = ids.new_empty((world * ids.shape[0], *ids.shape[1:]))
    dist.all_gather_into_tensor(out_s, scores.contiguous(), group=group)
    dist.all_gather_into_tensor(out_i, ids.contiguous(), group=group)
    return out_s.view(world, *scores.shape), out_i.view(world, *ids.shape)


def exchange_partials(o: torch.Tensor, lse: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather fp32 partial outputs ``(rows, D)`` and log-sum-exps ``(rows)``."""
    world = dist.get_world_size(group)
    out_o = o.new_empty((world * o.shape[0], *o.shape[1:]))
    out_l = lse.new_empty((world * lse.shape[0],))
    dist.all_gather_into_tensor(out_o, o.contiguous(), group=group)
    dist.all_gather_into_tensor(out_l, lse.contiguous(), group=group)
    return out_o.view(world, *o.shape), out_l.view(world, *lse.shape)


class ShardedQuestDecoder:
    """One rank's part of a sequence-sharded Quest decode step.

    ``cache`` holds this rank's pages; ``page_lo`` / ``page_hi`` (per sequence, global
    page ids) say which; ``last_here`` / ``sink_here`` whether this rank holds each
    sequence's last page / page 0 (all sequences alike).  ``exchange`` performs the
    all-gathers (default: ``torch.distributed`` on ``group``).
    """

    def __init__(self, cache: PagedKVCache, n_heads: int, topk: int, page_lo, page_hi, *, sink_pages: int = 0,
                 last_here: bool, sink_here: bool, scale: Optional[float] = None, group=None,
                 q_dtype: torch.dtype = torch.bfloat16):
        self.cache = cache
        self.n_heads = n_heads
        self.topk = topk
        self.group = group
        dev = cache.device
        self.page_lo = torch.as_tensor(page_lo, dtype=torch.int32, device=dev).reshape(cache.batch)
        self.page_hi = torch.as_tensor(page_hi, dtype=torch.int32, device=dev).reshape(cache.batch)
        self.local = QuestDecoder(cache, n_heads, topk, sink_pages=sink_pages if sink_here else 0, scale=scale,
                                  q_dtype=q_dtype, keep_scores=True, force_last=last_here)
        self.scale = self.local.scale
        b = cache.batch
        self.k = self.local.topk
        hkv = cache.n_kv_heads
        self.max_union = min((n_heads // hkv) * topk, cache.max_pages)
        self.union_ids = torch.empty(b, hkv, 1, self.max_union, dtype=torch.int32, device=dev)
        self.union_count = torch.empty(b, hkv, 1, dtype=torch.int32, device=dev)
        self.sel = torch.empty(b, n_heads, topk, dtype=torch.int32, device=dev)
        self.o_part = torch.empty(b, n_heads, 1, cache.head_dim, dtype=torch.float32, device=dev)
        self.lse_part = torch.empty(b, n_heads, 1, dtype=torch.float32, device=dev)
        self.out = torch.empty(b, n_heads, 1, cache.head_dim, dtype=q_dtype, device=dev)
        self._lists = L.Lists(self.union_ids.data_ptr(), L.I32, hkv, *self.union_ids.stride()[:3], self.max_union,
                              self.union_count.data_ptr(), *self.union_count.stride())

    def candidates(self, q: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Local top-K ``(scores, global ids)``, each ``(B, H_q, K)``."""
        sel = self.local.select(q)
        ids = sel.ids[:, :, 0, :]                                 # local pages, -1 padded
        scores = torch.gather(sel.scores[:, :, 0, :], -1, ids.clamp_min(0).long())
        gids = torch.where(ids >= 0, ids + self.page_lo.view(-1, 1, 1), torch.full_like(ids, -1))
        return scores.contiguous(), gids.contiguous()

    def merge(self, all_scores: torch.Tensor, all_ids: torch.Tensor) -> None:
        """Global top-K of the gathered candidates and this rank's share of the union."""
        r, b, hq, k = all_scores.shape
        L.check(L.lib().linattn_shard_merge(
            all_scores.data_ptr(), all_ids.data_ptr(), r, b, hq, k, self.topk, self.cache.n_kv_heads,
            self.page_lo.data_ptr(), self.page_hi.data_ptr(), self.cache.max_pages, self.sel.data_ptr(),
            self.union_ids.data_ptr(), self.union_count.data_ptr(), self.max_union, L.stream_of(all_scores)))

    def partial(self, q: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp32 ``(o, lse)`` of attention over this rank's selected pages."""
        need = L.lib().linattn_sparse_attention_workspace(q.shape[0], self.n_heads, 1, self.cache.head_dim, 1)
        ws = self.local.workspace if self.local.workspace.numel() * 4 >= need else \
            torch.empty((need + 3) // 4, dtype=torch.float32, device=q.device)
        status = L.status_word(q.device)
        L.check(L.lib().linattn_sparse_attention_out(
            q.data_ptr(), L.dtype_code(q), q.shape[0], self.n_heads, 1, L.strides4(q), self.cache.kv_desc(),
            self._lists, 0, 0, self.scale, self.o_part.data_ptr(), L.F32, L.strides4(self.o_part),
            self.lse_part.data_ptr(), 1, ws.data_ptr(), need, status.data_ptr(), L.stream_of(q)))
        return self.o_part, self.lse_part

    def combine(self, all_o: torch.Tensor, all_lse: torch.Tensor) -> torch.Tensor:
        """Log-sum-exp merge of the gathered partials into ``out (B, H_q, 1, D)``."""
        r = all_o.shape[0]
        rows = all_o[0].numel() // self.cache.head_dim
        L.check(L.lib().linattn_lse_combine(all_o.data_ptr(), all_lse.data_ptr(), r, rows, self.cache.head_dim,
                                            self.out.data_ptr(), L.dtype_code(self.out), None,
                                            L.stream_of(all_o)))
        return self.out

    def step(self, q: torch.Tensor, exchange_c=None, exchange_p=None) -> torch.Tensor:
        """One decode step: ``q (B, H_q, 1, D)`` (the same on every rank) -> ``o``."""
        exchange_c = exchange_c or (lambda s, i: exchange_candidates(s, i, self.group))
        exchange_p = exchange_p or (lambda o, l: exchange_partials(o, l, self.group))
        s, i = self.candidates(q)
        all_s, all_i = exchange_c(s, i)
        self.merge(all_s, all_i)
        o, lse = self.partial(q)
        all_o, all_l = exchange_p(o.view(-1, self.cache.head_dim), lse.view(-1))
        return self.combine(all_o, all_l)

