"""Paged KV pool with Quest metadata, and the allocation-free Quest decode step.

The reference has no physical paged cache (``src/linattn/kv/cache.py`` is a hit-rate
simulator); its only page layout is logical: page ``p`` of ``(b, h)`` is
``K[b, h, p*P:(p+1)*P]`` of a contiguous cache (``quest_pages.py:38-48``,
``c_attention.py:124-125``).  This module keeps that logical contract and stores it
B200-first:

* ``k_pool, v_pool [N_phys, H_kv, P, D]`` - each (page, head) is one contiguous
  ``P*D`` chunk (16 KiB in bf16 at P=64, D=128), moved by one TMA bulk copy;
* ``page_table int32 [B, max_pages]`` maps logical to physical pages;
* ``meta [B, H_kv, max_pages, 2, D]`` - Quest's channel bounds (min row, max row) in
  LOGICAL page order per sequence and kv head, so that scoring streams one
  contiguous block per (sequence, kv head) with large TMA copies (``meta_min`` /
  ``meta_max`` are views);
* fp8 e4m3 pools add ``k_scale/v_scale fp32 [N_phys, H_kv]`` (``kv/quant.py:90-93``
  applied per (page, head)); the metadata then bounds the dequantised keys, rounded
  outward to the metadata dtype.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import plan_splits, sparse_attention
from linattn_b200.quest_pages import DECODE_OFFSET, QuestSelection

__all__ = ["PagedKVCache", "QuestDecodeGraph", "QuestDecoder", "fused_select_smem", "plan_select_chunks"]


class PagedKVCache:
    """Physical paged KV pool (one per layer) with a host-side page allocator."""

    def __init__(self, batch: int, n_kv_heads: int, head_dim: int, page_size: int, max_pages: int, *,
                 num_phys_pages: Optional[int] = None, dtype: torch.dtype = torch.bfloat16,
                 meta_dtype: Optional[torch.dtype] = None, device="cuda"):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("PagedKVCache lives in device memory (cuda)")
        self.batch, self.n_kv_heads, self.head_dim, self.page_size = batch, n_kv_heads, head_dim, page_size
        self.max_pages = max_pages
        self.num_phys_pages = num_phys_pages or batch * max_pages
        self.fp8 = dtype in (torch.float8_e4m3fn, torch.uint8)
        self.dtype = dtype
        pool_dtype = torch.uint8 if self.fp8 else dtype
        shape = (self.num_phys_pages, n_kv_heads, page_size, head_dim)
        self.k_pool = torch.zeros(shape, dtype=pool_dtype, device=self.device)
        self.v_pool = torch.zeros(shape, dtype=pool_dtype, device=self.device)
        self.meta_dtype = meta_dtype or (torch.bfloat16 if self.fp8 else dtype)
        self.meta = torch.zeros(batch, n_kv_heads, max_pages, 2, head_dim, dtype=self.meta_dtype, device=self.device)
        self.meta_min = self.meta[..., 0, :]
        self.meta_max = self.meta[..., 1, :]
        if self.fp8:
            self.k_scale = torch.ones(self.num_phys_pages, n_kv_heads, dtype=torch.float32, device=self.device)
            self.v_scale = torch.ones_like(self.k_scale)
        else:
            self.k_scale = self.v_scale = None
        self.page_table = torch.full((batch, max_pages), -1, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.n_pages_b = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self._host_lens = [0] * batch
        self._host_table = [[] for _ in range(batch)]
        self._free = list(range(self.num_phys_pages - 1, -1, -1))

    # -- descriptors ---------------------------------------------------------------
    def kv_desc(self) -> L.KV:
        hk, p, d = self.n_kv_heads, self.page_size, self.head_dim
        return L.KV(self.k_pool.data_ptr(), self.v_pool.data_ptr(), 0, hk * p * d, p * d,
                    self.page_table.data_ptr(), self.max_pages, self.num_phys_pages,
                    L.ptr(self.k_scale), L.ptr(self.v_scale), hk, 1,
                    self.seq_lens.data_ptr(), 0, L.FP8E4M3 if self.fp8 else L.dtype_code(self.k_pool), p, d, hk,
                    self.num_phys_pages * hk * p)

    def meta_desc(self) -> L.Meta:
        hk, d, n = self.n_kv_heads, self.head_dim, self.max_pages
        return L.Meta(self.meta_min.data_ptr(), self.meta_max.data_ptr(), hk * n * 2 * d, 2 * d, n * 2 * d, None, 0,
                      0, L.dtype_code(self.meta), hk)

    # -- page allocation (host) ----------------------------------------------------
    def _ensure_pages(self, b: int, n_pages: int) -> None:
        table = self._host_table[b]
        if n_pages > self.max_pages:
            raise ValueError(f"sequence {b} needs {n_pages} pages > max_pages {self.max_pages}")
        new = []
        while len(table) < n_pages:
            if not self._free:
                raise RuntimeError("paged KV pool is full")
            phys = self._free.pop()
            table.append(phys)
            new.append(phys)
        if new:
            start = len(table) - len(new)
            self.page_table[b, start:len(table)] = torch.tensor(new, dtype=torch.int32, device=self.device)

    def set_page_table(self, table: torch.Tensor, seq_lens) -> None:
        """Install an externally built page table (e.g. a permutation) and lengths."""
        if table.shape != (self.batch, self.max_pages):
            raise ValueError("page table shape must be (batch, max_pages)")
        self.page_table.copy_(table.to(torch.int32))
        lens = [int(x) for x in seq_lens]
        self._host_lens = lens
        host = table.cpu().tolist()
        used = set()
        for b in range(self.batch):
            n = math.ceil(lens[b] / self.page_size)
            self._host_table[b] = [int(x) for x in host[b][:n]]
            used.update(self._host_table[b])
        self._free = [p for p in range(self.num_phys_pages - 1, -1, -1) if p not in used]
        self._sync_lens()

    def _sync_lens(self) -> None:
        lens = torch.tensor(self._host_lens, dtype=torch.int32)
        self.seq_lens.copy_(lens)
        self.n_pages_b.copy_((lens + self.page_size - 1) // self.page_size)

    # -- writes ----------------------------------------------------------------------
    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append ``(B, H_kv, T_new, D)`` keys/values to every sequence and fold them into
        the bounds of the pages they touch (``QuestAttention.push_kv`` +
        ``_refresh_pages``, ``src/linattn/variants/selection.py:176-201``): one
        ``linattn_paged_append`` launch after the host allocator has mapped any new
        pages.  16/32-bit pools only."""
        if self.fp8:
            raise NotImplementedError("fp8 pools are quantised a whole page at a time (fill)")
        L.require_cuda(k, v)
        b_, hk, tn, d = k.shape
        if (b_, hk, d) != (self.batch, self.n_kv_heads, self.head_dim) or v.shape != k.shape:
            raise ValueError("append shape mismatch")
        if tn == 0:
            return
        if k.stride(3) != 1:
            k = k.contiguous()
        if v.stride() != k.stride():
            v = v.contiguous()
            k = k.contiguous()
        for b in range(self.batch):
            self._ensure_pages(b, math.ceil((self._host_lens[b] + tn) / self.page_size))
        status = L.status_word(self.device)
        # start positions: the device lengths before the append (updated below, in
        # stream order after the kernel)
        L.check(L.lib().linattn_paged_append(
            self.kv_desc(), self.meta_desc(), self.batch, k.data_ptr(), v.data_ptr(), L.dtype_code(k),
            L.strides4(k), tn, self.seq_lens.data_ptr(), status.data_ptr(),
            torch.cuda.current_stream(self.device).cuda_stream))
        self._host_lens = [x + tn for x in self._host_lens]
        self._sync_lens()
        if L.strict():
            L.check_status(self.device)

    def fill(self, k: torch.Tensor, v: torch.Tensor, seq_lens, page_table: Optional[torch.Tensor] = None) -> None:
        """Write whole sequences: ``k, v (B, H_kv, T, D)`` (any float dtype) with
        ``seq_lens[b] <= T`` valid rows, through ``page_table (B, max_pages)`` (default:
        sequence b owns physical pages ``[b*max_pages, (b+1)*max_pages)``).  fp8 pools are
        quantised with one scale per (page, kv head): ``scale = max|x| / 448`` (clamped to
        1e-8), ``codes = e4m3(x / scale)`` (``src/linattn/kv/quant.py:90-93``).  The page
        metadata is rebuilt."""
        L.require_cuda(k, v)
        b_, hk, t, d = k.shape
        p = self.page_size
        if (b_, hk, d) != (self.batch, self.n_kv_heads, self.head_dim) or t > self.max_pages * p:
            raise ValueError("fill shape mismatch")
        if page_table is None:
            page_table = torch.arange(self.batch * self.max_pages, dtype=torch.int32).view(self.batch, self.max_pages)
        n = -(-t // p)
        pad = n * p - t
        kp = torch.nn.functional.pad(k.float(), (0, 0, 0, pad)).view(b_, hk, n, p, d).transpose(1, 2)
        vp = torch.nn.functional.pad(v.float(), (0, 0, 0, pad)).view(b_, hk, n, p, d).transpose(1, 2)
        phys = page_table[:, :n].to(self.device).long().reshape(-1)
        kp = kp.reshape(-1, hk, p, d)
        vp = vp.reshape(-1, hk, p, d)
        if self.fp8:
            for src, pool, sc in ((kp, self.k_pool, self.k_scale), (vp, self.v_pool, self.v_scale)):
                amax = src.abs().amax(dim=(2, 3)).clamp_min(1e-8)
                scale = amax / torch.full_like(amax, 448.0)  # true division, not * (1/448)
                codes = (src / scale[:, :, None, None]).to(torch.float8_e4m3fn).view(torch.uint8)
                pool[phys] = codes
                sc[phys] = scale
        else:
            self.k_pool[phys] = kp.to(self.k_pool.dtype)
            self.v_pool[phys] = vp.to(self.v_pool.dtype)
        self.set_page_table(page_table, seq_lens)
        self.refresh_meta()

    def refresh_meta(self, first_page: Optional[torch.Tensor] = None) -> None:
        """Recompute page bounds for pages ``[first_page[b], n_pages_b)`` (all if None)."""
        status = L.status_word(self.device)
        kv, meta = self.kv_desc(), self.meta_desc()
        L.check(L.lib().linattn_paged_page_bounds(kv, self.batch, L.ptr(first_page), self.max_pages, meta,
                                                  status.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))
        if L.strict():
            L.check_status(self.device)


def fused_select_smem(chunk: int, g: int, topk: int, d: int, mma: bool, cand: bool) -> int:
    """Shared memory of the fused selection kernel for `chunk` pages per CTA: the
    tensor-core path (q and metadata of one 16-bit type) streams 4 (single-CTA form) or
    2 (candidates form) stages of 64 pages, the CUDA-core path 8 or 4 stages of 32."""
    rest = g * chunk * 4 + 8 * 256 * 4 + ((chunk + 31) // 32) * 4 + 8 * 2 * topk * 4
    if mma:
        return 1024 + (2 if cand else 4) * 2 * d * 64 * 2 + rest
    return (4 if cand else 8) * 32 * 2 * d * 2 + rest


_SMEM_MAX = 220 * 1024
_SMEM_TWO_PER_SM = 113 * 1024


def plan_select_chunks(n: int, g: int, topk: int, d: int, units: int, device, chunks: Optional[int] = None,
                       ranks: int = 1, mma: bool = True, cand_only: bool = False, premerge: bool = False):
    """(pages per CTA, chunks) for the fused selection over `n` pages and `units`
    (sequence, kv head) pairs.  One chunk (the single-CTA form, no merge) when the
    pairs alone fill the GPU and the whole sequence's scores fit in shared memory;
    else chunks small enough for two CTAs per SM and numerous enough for two CTAs per
    SM.  Returns 0 chunks when the merge's bound (64 blocks and 4096 candidates per head
    across the chunks of all `ranks`; with `premerge`, each rank first merges its own chunks, so
    across the chunks of one rank and across the ranks) or shared memory rules the
    fused kernel out."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    if chunks is None:
        if not cand_only and units >= 0.8 * sms and fused_select_smem(n, g, topk, d, mma, False) <= _SMEM_MAX:
            chunks = 1
        else:
            cap = 64
            while cap * 2 <= n and fused_select_smem(cap * 2, g, topk, d, mma, True) <= _SMEM_TWO_PER_SM:
                cap *= 2
            chunks = max(-(-n // cap), min(-(-2 * sms // max(1, units)), -(-n // 128)))
    chunks = max(1, min(chunks, n))
    chunk = -(-n // chunks)
    single = chunks == 1 and not cand_only
    while fused_select_smem(chunk, g, topk, d, mma, not single) > _SMEM_MAX and chunk > 32:
        chunk = -(-chunk // 2)
        single = False
    chunks = -(-n // chunk)
    n_blocks = max(chunks, ranks) if premerge else chunks * ranks  # blocks of topk one merge takes
    if n_blocks * topk > 4096 or n_blocks > 64 or fused_select_smem(chunk, g, topk, d, mma, not single) > _SMEM_MAX:
        return chunk, 0
    return chunk, chunks


class QuestDecoder:
    """One Quest decode step over a :class:`PagedKVCache`, with every buffer allocated
    once: page scores -> top-k + GQA union -> sparse attention (split-KV + merge).

    ``step(q)`` takes ``q (B, H_q, 1, D)`` (one new token per sequence, at position
    ``seq_len_b - 1``) and returns ``o (B, H_q, 1, D)`` in q's dtype.  The budget is
    ``topk`` pages per query head including the forced pages (own page and
    ``sink_pages`` leading pages), as in ``page_select_torch``.
    """

    def __init__(self, cache: PagedKVCache, n_heads: int, topk: int, *, sink_pages: int = 0,
                 scale: Optional[float] = None, gqa_union: bool = True, n_splits: Optional[int] = None,
                 q_dtype: torch.dtype = torch.bfloat16, keep_scores: bool = False, force_last: bool = True,
                 select_chunks: Optional[int] = None):
        self.cache = cache
        # False on a shard of a sequence-sharded cache that does not hold the query's page
        self.force_last = force_last
        self.n_heads = n_heads
        self.group = n_heads // cache.n_kv_heads if gqa_union else 1
        self.topk = max(1, min(topk, cache.max_pages))
        self.sink_pages = sink_pages
        self.scale = scale if scale is not None else 1.0 / math.sqrt(cache.head_dim)
        dev = cache.device
        b, n = cache.batch, cache.max_pages
        group_size = n_heads // cache.n_kv_heads
        # fused selection: one CTA per (sequence, kv head), or per (sequence, kv head,
        # chunk of pages) followed by the merge of the chunks' candidates when the
        # sequence is long or the batch too small to fill the GPU
        self.fused = (gqa_union and group_size in (1, 2, 4, 8) and cache.head_dim in (64, 128)
                      and cache.meta_dtype in (torch.float16, torch.bfloat16))
        self.chunks = 1
        if self.fused:
            mma = q_dtype == cache.meta_dtype
            self.chunk_pages, self.chunks = plan_select_chunks(n, group_size, self.topk, cache.head_dim,
                                                               b * cache.n_kv_heads, dev, select_chunks, mma=mma)
            self.fused = self.chunks >= 1  # else the unfused path (scores, then top-k)
        self.keep_scores = keep_scores or not self.fused
        self.scores = torch.empty(b, n_heads, 1, n, dtype=torch.float32, device=dev) if self.keep_scores else None
        if self.fused and self.chunks > 1:
            # candidates (chunk, [scores | ids], B, H_q, topk) and the zero page base
            self.cand = torch.empty(self.chunks, 2, b, n_heads, self.topk, dtype=torch.int32, device=dev)
            self.page_zero = torch.zeros(b, dtype=torch.int32, device=dev)
        self.ids = torch.empty(b, n_heads, 1, self.topk, dtype=torch.int32, device=dev)
        self.max_union = min(self.group * self.topk, n)
        n_lists = n_heads // self.group
        self.union_ids = torch.empty(b, n_lists, 1, self.max_union, dtype=torch.int32, device=dev)
        self.union_count = torch.empty(b, n_lists, 1, dtype=torch.int32, device=dev)
        self.union_tokens = torch.empty_like(self.union_count)
        self.out = torch.empty(b, n_heads, 1, cache.head_dim, dtype=q_dtype, device=dev)
        kv_code = L.FP8E4M3 if cache.fp8 else L.dtype_code(cache.k_pool)
        q_code = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}[q_dtype]
        self.n_splits = n_splits or plan_splits(b, n_heads, 1, cache.head_dim, kv_code, q_code, n_lists,
                                                self.max_union, cache.page_size, dev)
        need = L.lib().linattn_sparse_attention_workspace(b, n_heads, 1, cache.head_dim, self.n_splits)
        self.workspace = torch.empty(max(1, (need + 3) // 4), dtype=torch.float32, device=dev)
        self._lists = L.Lists(self.union_ids.data_ptr(), L.I32, n_lists, *self.union_ids.stride()[:3],
                              self.max_union, self.union_count.data_ptr(), *self.union_count.stride())

    def select(self, q: torch.Tensor) -> QuestSelection:
        c = self.cache
        dev = c.device
        status = L.status_word(dev)
        stream = L.stream_of(q)
        b, hq, tq, d = q.shape
        lib = L.lib()
        if self.fused and self.chunks > 1:
            bhk = b * hq * self.topk
            L.check(lib.linattn_quest_decode_candidates(
                q.data_ptr(), L.dtype_code(q), b, hq, d, L.strides4(q), c.meta.data_ptr(), L.dtype_code(c.meta),
                c.n_kv_heads, c.max_pages, c.n_pages_b.data_ptr(), self.topk, self.sink_pages, int(self.force_last),
                self.chunk_pages, None, self.cand.data_ptr(), self.cand[:, 1].data_ptr(), 2 * bhk,
                L.ptr(self.scores), status.data_ptr(), stream))
            L.check(lib.linattn_shard_merge(
                self.cand.data_ptr(), self.cand[:, 1].data_ptr(), self.chunks, b, hq, self.topk, 2 * bhk, self.topk,
                c.n_kv_heads, self.page_zero.data_ptr(), c.n_pages_b.data_ptr(), c.max_pages, self.ids.data_ptr(), None,
                self.union_ids.data_ptr(), self.union_count.data_ptr(), self.max_union, c.seq_lens.data_ptr(),
                c.page_size, self.union_tokens.data_ptr(), stream))
            return QuestSelection(self.ids, self.scores, self.union_ids, self.union_count, self.union_tokens)
        if self.fused:
            L.check(lib.linattn_quest_decode_select(
                q.data_ptr(), L.dtype_code(q), b, hq, d, L.strides4(q), c.meta.data_ptr(), L.dtype_code(c.meta),
                c.n_kv_heads, c.max_pages, c.n_pages_b.data_ptr(), c.seq_lens.data_ptr(), c.page_size, self.topk,
                self.sink_pages, int(self.force_last), self.ids.data_ptr(), L.ptr(self.scores),
                self.union_ids.data_ptr(),
                self.union_count.data_ptr(), self.max_union, self.union_tokens.data_ptr(), status.data_ptr(), stream))
            return QuestSelection(self.ids, self.scores, self.union_ids, self.union_count, self.union_tokens)
        L.check(lib.linattn_quest_scores(q.data_ptr(), L.dtype_code(q), b, hq, tq, d, L.strides4(q), c.meta_desc(),
                                         c.page_size, c.max_pages, DECODE_OFFSET, self.sink_pages,
                                         c.n_pages_b.data_ptr(), self.scores.data_ptr(), status.data_ptr(), stream))
        L.check(lib.linattn_page_topk(self.scores.data_ptr(), b, hq, tq, c.max_pages, self.topk,
                                      c.n_pages_b.data_ptr(), None, self.ids.data_ptr(), self.group,
                                      self.union_ids.data_ptr(), self.union_count.data_ptr(), self.max_union,
                                      self.union_tokens.data_ptr(), c.page_size, DECODE_OFFSET,
                                      c.seq_lens.data_ptr(), 0, status.data_ptr(), stream))
        return QuestSelection(self.ids, self.scores, self.union_ids, self.union_count, self.union_tokens)

    def attend(self, q: torch.Tensor) -> torch.Tensor:
        sparse_attention(q, self.cache.kv_desc(), self._lists, causal=False, scale=self.scale, out=self.out,
                         n_splits=self.n_splits, workspace=self.workspace)
        return self.out

    def step(self, q: torch.Tensor) -> torch.Tensor:
        if q.shape != (self.cache.batch, self.n_heads, 1, self.cache.head_dim):
            raise ValueError(f"q must be (B, H_q, 1, D) = {(self.cache.batch, self.n_heads, 1, self.cache.head_dim)}")
        self.select(q)
        out = self.attend(q)
        if L.strict():
            L.check_status(self.cache.device)
        return out

    def graph(self) -> "QuestDecodeGraph":
        """The decode step as one CUDA graph with pinned host input and output."""
        return QuestDecodeGraph(self)


class QuestDecodeGraph:
    """A :class:`QuestDecoder` step captured once as a CUDA graph: the copy of q from a
    pinned host buffer, the selection and attention launches, and the copy of o back
    to a pinned host buffer.  ``run(q_host)`` copies ``q_host`` (B, H_q, 1, D) into the
    staging buffer, replays the graph on the current stream and returns the pinned
    output, valid once the stream is synchronised (stage the next q only after that).
    The graph holds the cache's buffer addresses, not their contents, so appends
    between replays are seen (the cache must not be re-allocated)."""

    def __init__(self, dec: QuestDecoder):
        c = dec.cache
        if L.strict():
            raise RuntimeError("QuestDecodeGraph: strict mode synchronises inside the step and cannot be captured")
        self.dec = dec
        shape = (c.batch, dec.n_heads, 1, c.head_dim)
        self.q_host = torch.empty(shape, dtype=dec.out.dtype, pin_memory=True)
        self.o_host = torch.empty(shape, dtype=dec.out.dtype, pin_memory=True)
        self.q_dev = torch.zeros(shape, dtype=dec.out.dtype, device=c.device)
        # one eager step on a side stream first: status word, tensor maps and kernel
        # attributes are set up outside the capture
        side = torch.cuda.Stream(c.device)
        side.wait_stream(torch.cuda.current_stream(c.device))
        with torch.cuda.stream(side):
            dec.step(self.q_dev)
        torch.cuda.current_stream(c.device).wait_stream(side)
        torch.cuda.synchronize(c.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.q_dev.copy_(self.q_host, non_blocking=True)
            out = dec.step(self.q_dev)
            self.o_host.copy_(out, non_blocking=True)

    def run(self, q_host: Optional[torch.Tensor] = None) -> torch.Tensor:
        if q_host is not None:
            self.q_host.copy_(q_host)
        self.graph.replay()
        return self.o_host
