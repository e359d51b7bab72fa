"""Sequence-sharded Quest decode across GPUs (the million-token configuration).

Every rank holds a contiguous slice of each sequence's KV pages (``PagedKVCache`` of
the slice, pages ``[page_lo_b, page_hi_b)`` of sequence ``b``).  One decode step:

1. local selection (the candidates form of the fused Quest kernel) gives each query
   head the top-K pages of each chunk of the shard with their scores; only the rank
   holding a sequence's last page forces it in, only the rank holding page 0 forces
   the sink pages; with several ranks the shard merges its chunks into its own top-K
   (``linattn_shard_merge`` without the union), one sorted block of K per head;
2. the (score, global page) candidates are all-gathered (rank-major): R blocks of K
   per head, whatever the number of chunks;
3. every rank takes the same global top-K per head (``linattn_shard_merge``: score
   desc, lowest page on ties, as the single-cache selection) and keeps the GQA union
   of the selected pages it owns;
4. attention over those pages gives fp32 partial ``(o, lse)`` (``lse = -inf`` for a rank
   that owns none of them);
5. the partials are all-gathered and merged by the log-sum-exp combine kernel.

Each exchange is one ``torch.distributed.all_gather_into_tensor`` of one packed buffer
per rank (``exchange_packed``; NCCL over NVLink between GPUs, any backend for testing
the layout on CPU).  ``exchange_candidates`` / ``exchange_partials`` gather unpacked
tensors for callers that keep them apart.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import plan_splits
from linattn_b200.paged import PagedKVCache, plan_select_chunks

__all__ = ["ShardedQuestDecoder", "exchange_candidates", "exchange_packed", "exchange_partials", "shard_page_ranges"]


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


def exchange_packed(buf: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one rank's contiguous buffer into ``(R, *buf.shape)`` (rank-major)."""
    world = dist.get_world_size(group)
    out = buf.new_empty((world * buf.shape[0], *buf.shape[1:]))
    dist.all_gather_into_tensor(out, buf.contiguous(), group=group)
    return out.view(world, *buf.shape)


class ShardedQuestDecoder:
    """One rank's part of a sequence-sharded Quest decode step.

    ``cache`` holds this rank's pages; ``page_lo`` / ``page_hi`` (per sequence, global
    page ids) say which; ``last_here`` / ``sink_here`` whether this rank holds each
    sequence's last page / page 0 (all sequences alike); ``n_ranks`` is the number of
    shards (default: the process group's size).

    Local selection is the candidates form of the fused Quest kernel: the shard's pages
    are cut into ``chunks`` chunks and each chunk proposes every head's top-``topk``
    pages with their scores.  Each exchange moves ONE buffer per rank: the candidates
    as ``cand (chunks, 2, B, H_q, topk)`` int32 (fp32 score bits, then global page ids)
    and the partials as ``part (rows * D + rows)`` fp32 (``o`` rows, then their lse), so
    a step costs two all-gathers; the merge and combine kernels read the gathered
    buffers in place through their rank strides.  ``select_chunks`` / ``n_splits``
    override the planned chunk count of the local selection / the split-KV count of
    the local attention.
    """

    def __init__(self, cache: PagedKVCache, n_heads: int, topk: int, page_lo, page_hi, *, sink_pages: int = 0,
                 last_here: bool, sink_here: bool, scale: Optional[float] = None, group=None,
                 q_dtype: torch.dtype = torch.bfloat16, n_ranks: Optional[int] = None,
                 select_chunks: Optional[int] = None, n_splits: Optional[int] = None):
        self.cache = cache
        self.n_heads = n_heads
        self.topk = topk
        self.group = group
        self.sink_pages = sink_pages if sink_here else 0
        self.force_last = bool(last_here)
        self.scale = scale if scale is not None else 1.0 / math.sqrt(cache.head_dim)
        dev = cache.device
        b, hkv, d = cache.batch, cache.n_kv_heads, cache.head_dim
        g = n_heads // hkv
        if n_ranks is None:
            n_ranks = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.n_ranks = n_ranks
        if not (n_heads % hkv == 0 and g in (1, 2, 4, 8) and d in (64, 128)
                and cache.meta_dtype in (torch.float16, torch.bfloat16)):
            raise NotImplementedError("sharded decode needs f16/bf16 page metadata, head_dim 64 or 128 and a GQA "
                                      "group of 1, 2, 4 or 8 query heads")
        self.chunk_pages, self.chunks = plan_select_chunks(cache.max_pages, g, topk, d, b * hkv, dev, select_chunks,
                                                           ranks=n_ranks, mma=q_dtype == cache.meta_dtype,
                                                           cand_only=True, premerge=n_ranks > 1)
        if self.chunks == 0:
            raise NotImplementedError(f"sharded decode: {n_ranks} ranks x topk {topk} exceed the merge kernel's 4096 "
                                      "candidates per head")
        self.page_lo = torch.as_tensor(page_lo, dtype=torch.int32, device=dev).reshape(b)
        self.page_hi = torch.as_tensor(page_hi, dtype=torch.int32, device=dev).reshape(b)
        self.max_union = min(g * topk, cache.max_pages)
        self.union_ids = torch.empty(b, hkv, 1, self.max_union, dtype=torch.int32, device=dev)
        self.union_count = torch.empty(b, hkv, 1, dtype=torch.int32, device=dev)
        self.union_tokens = torch.empty(b, hkv, 1, dtype=torch.int32, device=dev)
        self.sel = torch.empty(b, n_heads, topk, dtype=torch.int32, device=dev)
        self.cand = torch.empty(self.chunks, 2, b, n_heads, topk, dtype=torch.int32, device=dev)
        # with several ranks each one first merges its own chunks into one sorted block of
        # K ([score bits | ids], the same layout), so the exchange and the global merge
        # see R blocks instead of R * chunks
        self.premerge = n_ranks > 1 and self.chunks > 1
        self.block = torch.empty(2, b, n_heads, topk, dtype=torch.int32, device=dev) if self.premerge else None
        rows = b * n_heads
        self.rows = rows
        self.part = torch.empty(rows * d + rows, dtype=torch.float32, device=dev)
        self.o_part = self.part[:rows * d].view(b, n_heads, 1, d)
        self.lse_part = self.part[rows * d:].view(b, n_heads, 1)
        self.out = torch.empty(b, n_heads, 1, d, dtype=q_dtype, device=dev)
        self._lists = L.Lists(self.union_ids.data_ptr(), L.I32, hkv, *self.union_ids.stride()[:3], self.max_union,
                              self.union_count.data_ptr(), *self.union_count.stride())
        kv_code = L.FP8E4M3 if cache.fp8 else L.dtype_code(cache.k_pool)
        q_code = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}[q_dtype]
        self.n_splits = n_splits or plan_splits(b, n_heads, 1, d, kv_code, q_code, hkv, self.max_union,
                                                cache.page_size, dev)
        self._ws_bytes = L.lib().linattn_sparse_attention_workspace(b, n_heads, 1, d, self.n_splits)
        self._ws = torch.empty(max(1, (self._ws_bytes + 3) // 4), dtype=torch.float32, device=dev)

    def candidates(self, q: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Local candidates ``(scores, global ids)``, each ``(chunks, B, H_q, topk)``
        (views of ``cand``)."""
        c = self.cache
        b, hq, _, d = q.shape
        status = L.status_word(q.device)
        bhk = b * hq * self.topk
        L.check(L.lib().linattn_quest_decode_candidates(
            q.data_ptr(), L.dtype_code(q), b, hq, d, L.strides4(q), c.meta.data_ptr(), L.dtype_code(c.meta),
            c.n_kv_heads, c.max_pages, c.n_pages_b.data_ptr(), self.topk, self.sink_pages, int(self.force_last),
            self.chunk_pages, self.page_lo.data_ptr(), self.cand.data_ptr(), self.cand[:, 1].data_ptr(), 2 * bhk,
            None, status.data_ptr(), L.stream_of(q)))
        if self.premerge:
            L.check(L.lib().linattn_shard_merge(
                self.cand.data_ptr(), self.cand[:, 1].data_ptr(), self.chunks, b, hq, self.topk, 2 * bhk, self.topk,
                c.n_kv_heads, self.page_lo.data_ptr(), self.page_hi.data_ptr(), c.max_pages,
                self.block[1].data_ptr(), self.block[0].data_ptr(), None, None, 0, None, 0, None, L.stream_of(q)))
            return self.block[0].view(torch.float32).unsqueeze(0), self.block[1].unsqueeze(0)
        return self.cand[:, 0].view(torch.float32), self.cand[:, 1]

    @property
    def exchange_buf(self) -> torch.Tensor:
        """The candidates buffer a step exchanges: ``(2, B, H_q, topk)`` after the
        pre-merge, else ``cand (chunks, 2, B, H_q, topk)``."""
        return self.block if self.premerge else self.cand

    def merge(self, all_scores: torch.Tensor, all_ids: torch.Tensor) -> None:
        """Global top-``topk`` of the gathered candidates ``(R, B, H_q, K)`` (R blocks,
        rank-major; the block stride may exceed ``B*H_q*K``) and this rank's share of
        the union."""
        r, b, hq, k = all_scores.shape
        if not (all_scores[0].is_contiguous() and all_ids[0].is_contiguous()) or \
                all_scores.stride(0) != all_ids.stride(0) or all_scores.dtype != torch.float32:
            raise ValueError("merge: per-block candidates must be contiguous fp32 / int32 with one block stride")
        L.check(L.lib().linattn_shard_merge(
            all_scores.data_ptr(), all_ids.data_ptr(), r, b, hq, k, all_scores.stride(0) if r > 1 else 0, self.topk,
            self.cache.n_kv_heads, self.page_lo.data_ptr(), self.page_hi.data_ptr(), self.cache.max_pages,
            self.sel.data_ptr(), None, self.union_ids.data_ptr(), self.union_count.data_ptr(), self.max_union,
            self.cache.seq_lens.data_ptr(), self.cache.page_size, self.union_tokens.data_ptr(),
            L.stream_of(all_scores)))

    def merge_packed(self, allc: torch.Tensor) -> None:
        """``merge`` over gathered ``exchange_buf`` buffers ``(R, [chunks,] 2, B, H_q, topk)``."""
        blocks = allc.reshape(-1, *allc.shape[-4:])  # (R * chunks, 2, B, H_q, topk)
        self.merge(blocks[:, 0].view(torch.float32), blocks[:, 1])

    def partial(self, q: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp32 ``(o, lse)`` of attention over this rank's selected pages (views of ``part``)."""
        status = L.status_word(q.device)
        L.check(L.lib().linattn_sparse_attention_out(
            q.data_ptr(), L.dtype_code(q), q.shape[0], self.n_heads, 1, L.strides4(q), self.cache.kv_desc(),
            self._lists, 0, 0, self.scale, self.o_part.data_ptr(), L.F32, L.strides4(self.o_part),
            self.lse_part.data_ptr(), self.n_splits, self._ws.data_ptr(), self._ws_bytes, status.data_ptr(),
            L.stream_of(q)))
        return self.o_part, self.lse_part

    def combine(self, all_o: torch.Tensor, all_lse: torch.Tensor) -> torch.Tensor:
        """Log-sum-exp merge of the gathered partials ``all_o (R, rows, D)``, ``all_lse
        (R, rows)`` (rank strides may exceed the dense ones) into ``out (B, H_q, 1, D)``."""
        r = all_o.shape[0]
        d = self.cache.head_dim
        if not (all_o[0].is_contiguous() and all_lse[0].is_contiguous()):
            raise ValueError("combine: per-rank blocks must be contiguous")
        L.check(L.lib().linattn_lse_combine_strided(
            all_o.data_ptr(), all_o.stride(0) if r > 1 else 0, all_lse.data_ptr(), all_lse.stride(0) if r > 1 else 0,
            r, self.rows, d, self.out.data_ptr(), L.dtype_code(self.out), None, L.stream_of(all_o)))
        return self.out

    def combine_packed(self, allp: torch.Tensor) -> torch.Tensor:
        """``combine`` over gathered ``part`` buffers ``(R, rows * D + rows)``."""
        rd = self.rows * self.cache.head_dim
        return self.combine(allp[:, :rd].view(-1, self.rows, self.cache.head_dim), allp[:, rd:])

    def step(self, q: torch.Tensor, exchange=None) -> torch.Tensor:
        """One decode step: ``q (B, H_q, 1, D)`` (the same on every rank) -> ``o``.
        ``exchange(buf) -> (R, *buf.shape)`` gathers one buffer from every rank
        (default: ``exchange_packed`` on the process group)."""
        exchange = exchange or (lambda t: exchange_packed(t, self.group))
        self.candidates(q)
        self.merge_packed(exchange(self.exchange_buf))
        self.partial(q)
        return self.combine_packed(exchange(self.part))
