"""Quest page metadata, scoring and top-k selection on the B200.

Same names, arguments and results as ``src/linattn/kernels/triton/quest_pages.py``
(``page_bounds_torch`` / ``page_select_torch`` / ``page_select_triton``), computed
by the sm_100a kernels of ``liblinattn_b200.so``:

* ``page_bounds(k, page_size)`` -> ``(mins, maxs)`` (``quest_pages.py:38-48``);
* ``page_select(q, mins, maxs, page_size, topk, offset=0)`` -> ``(ids int64, scores fp32)``
  (``quest_pages.py:57-78``; the own page is forced per query row as in
  ``src/linattn/variants/selection.py:220-230``, which equals the operator at
  ``T_q == 1``).  Ties are broken by the lowest page index.
* ``quest_select(...)`` additionally returns the GQA union per kv head
  (``selection.py:232-235``) as ascending page lists, which the attention kernel
  consumes without a host round trip.

The metadata may carry one head per query head (the reference operator) or one per
kv head (GQA; query head ``h`` reads metadata head ``h // (H_q / H_m)``).
"""

from __future__ import annotations

from typing import NamedTuple, Optional, Tuple

import torch

from linattn_b200 import _lib as L

__all__ = ["page_bounds", "page_select", "quest_select", "QuestSelection", "DECODE_OFFSET"]

# offset used for decode against ragged sequences: every page below the sequence's
# page count is visible and the own page is the last one
DECODE_OFFSET = 1 << 60


def _meta_contig(mins: torch.Tensor, maxs: torch.Tensor) -> L.Meta:
    if mins.shape != maxs.shape or mins.dtype != maxs.dtype:
        raise ValueError("mins and maxs must have the same shape and dtype")
    if mins.stride(-1) != 1 or maxs.stride() != mins.stride():
        raise ValueError("mins/maxs need unit stride on the channel axis and identical strides")
    sb, sh, sp, _ = mins.stride()
    return L.Meta(mins.data_ptr(), maxs.data_ptr(), sb, sp, sh, None, 0, 0, L.dtype_code(mins), mins.shape[1])


def page_bounds(k: torch.Tensor, page_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Channel-wise min/max per page: ``(B,H_kv,T,D) -> (B,H_kv,n_pages,D)`` (same dtype).

    Replaces ``page_bounds_torch`` (``quest_pages.py:38-48``); rows past ``T`` in the
    tail page are ignored, as the reference's +/-inf padding makes them.
    """
    dev = L.require_cuda(k)
    if k.dim() != 4:
        raise ValueError("k must have shape (B, H_kv, T, D)")
    if page_size <= 0:
        raise ValueError("page_size must be positive")
    b, h, t, d = k.shape
    n = (t + page_size - 1) // page_size
    mins = torch.empty(b, h, n, d, dtype=k.dtype, device=dev)
    maxs = torch.empty_like(mins)
    L.check(L.lib().linattn_page_bounds(k.data_ptr(), L.dtype_code(k), b, h, t, d, L.strides4(k), page_size,
                                        mins.data_ptr(), maxs.data_ptr(), L.stream_of(k)))
    return mins, maxs


class QuestSelection(NamedTuple):
    ids: torch.Tensor  # (B, H_q, T_q, k) int64/int32, score-descending, -1 padded
    scores: torch.Tensor  # (B, H_q, T_q, n_pages) fp32, masked (-inf) / forced (+inf)
    union_ids: Optional[torch.Tensor]  # (B, H_q/group, T_q, max_union) int32 ascending, -1 padded
    union_count: Optional[torch.Tensor]  # (B, H_q/group, T_q) int32
    union_tokens: Optional[torch.Tensor]  # (B, H_q/group, T_q) int32: tokens those pages hold (causal)


def quest_select(q: torch.Tensor, meta: L.Meta, *, page_size: int, n_pages: int, topk: int, offset: int = 0,
                 sink_pages: int = 0, group: int = 1, n_pages_b: Optional[torch.Tensor] = None,
                 seq_lens: Optional[torch.Tensor] = None, seq_len: int = 0, ids_dtype=torch.int64,
                 with_union: bool = True, scores_out: Optional[torch.Tensor] = None) -> QuestSelection:
    """Score every page, keep the top-k per query head and (optionally) the union per
    group of ``group`` query heads.  ``meta`` describes contiguous or paged metadata."""
    dev = L.require_cuda(q)
    b, hq, tq, d = q.shape
    stream = L.stream_of(q)
    status = L.status_word(dev)
    scores = scores_out if scores_out is not None else torch.empty(b, hq, tq, n_pages, dtype=torch.float32,
                                                                   device=dev)
    L.check(L.lib().linattn_quest_scores(q.data_ptr(), L.dtype_code(q), b, hq, tq, d, L.strides4(q),
                                         meta, page_size, n_pages, offset, sink_pages, L.ptr(n_pages_b),
                                         scores.data_ptr(), status.data_ptr(), stream))
    k = max(1, min(topk, n_pages))
    ids = torch.empty(b, hq, tq, k, dtype=ids_dtype, device=dev)
    union_ids = union_count = union_tokens = None
    if with_union:
        if hq % group:
            raise ValueError("group must divide the number of query heads")
        max_union = min(group * k, n_pages)
        union_ids = torch.empty(b, hq // group, tq, max_union, dtype=torch.int32, device=dev)
        union_count = torch.empty(b, hq // group, tq, dtype=torch.int32, device=dev)
        union_tokens = torch.empty_like(union_count)
    else:
        max_union = 0
    L.check(L.lib().linattn_page_topk(
        scores.data_ptr(), b, hq, tq, n_pages, k, L.ptr(n_pages_b),
        ids.data_ptr() if ids_dtype == torch.int64 else None,
        ids.data_ptr() if ids_dtype == torch.int32 else None,
        group if with_union else 1, L.ptr(union_ids), L.ptr(union_count), max_union, L.ptr(union_tokens),
        page_size, offset, L.ptr(seq_lens), seq_len, status.data_ptr(), stream))
    if L.strict():
        L.check_status(dev)
    return QuestSelection(ids, scores, union_ids, union_count, union_tokens)


def page_select(q: torch.Tensor, mins: torch.Tensor, maxim: torch.Tensor, page_size: int, topk: int, *,
                offset: int = 0, sink_pages: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k page ids per query plus the page scores.

    Replaces ``page_select_torch`` / ``page_select_triton``
    (``src/linattn/kernels/triton/quest_pages.py:57-78``, ``:145-161``).  ``q``:
    ``(B,H,T_q,D)``; ``mins``/``maxim``: ``(B,H_m,n_pages,D)`` with ``H_m`` dividing
    ``H``.  Returns ``ids (B,H,T_q,k) int64`` sorted by descending score (ties: lowest
    page index) and ``scores (B,H,T_q,n_pages) float32`` with invisible pages at -inf
    and each query's own page (plus ``sink_pages`` leading pages) at +inf.
    """
    L.require_cuda(q, mins, maxim)
    if q.dim() != 4 or mins.dim() != 4:
        raise ValueError("q must be (B,H,T_q,D) and mins/maxs (B,H_m,n_pages,D)")
    if mins.shape[0] != q.shape[0] or mins.shape[-1] != q.shape[-1]:
        raise ValueError("batch / head_dim mismatch between q and the page metadata")
    meta = _meta_contig(mins, maxim)
    sel = quest_select(q, meta, page_size=page_size, n_pages=mins.shape[2], topk=topk, offset=offset,
                       sink_pages=sink_pages, with_union=False)
    return sel.ids, sel.scores
