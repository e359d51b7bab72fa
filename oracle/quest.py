"""Quest page metadata, page scores and top-k page selection (numpy restatement).

Test infrastructure only (see ``oracle/__init__.py``).  Scores are accumulated in
float64: every product of two fp16/bf16/fp32 values is exact in float64, so the
oracle score is the exact bound up to one float64 rounding of a 128-term sum.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "page_bounds",
    "page_scores",
    "page_select",
    "topk_lowest_index",
    "gqa_union",
    "quest_effective_mask",
]


def page_bounds(k: np.ndarray, page_size: int):
    """Channel-wise min/max per page, ``(B,H,T,D) -> (B,H,n_pages,D)``.

    Follows ``src/linattn/kernels/triton/quest_pages.py:38-48``: the tail page is
    padded with +inf (for the min) and -inf (for the max) so the padding never wins.
    Min/max is exact, so the result keeps the input dtype.
    """
    b, h, t, d = k.shape
    n_pages = (t + page_size - 1) // page_size
    pad = n_pages * page_size - t
    lo = np.concatenate([k, np.full((b, h, pad, d), np.inf, dtype=k.dtype)], axis=2)
    hi = np.concatenate([k, np.full((b, h, pad, d), -np.inf, dtype=k.dtype)], axis=2)
    mins = lo.reshape(b, h, n_pages, page_size, d).min(axis=3)
    maxs = hi.reshape(b, h, n_pages, page_size, d).max(axis=3)
    return mins, maxs


def page_scores(q: np.ndarray, mins: np.ndarray, maxs: np.ndarray) -> np.ndarray:
    """Upper-bound page scores ``s[b,h,t,p] = sum_d max(q_d*min_d, q_d*max_d)``.

    ``src/linattn/kernels/triton/quest_pages.py:51-54`` and, for the GQA head
    mapping (query head ``h`` reads kv head ``h // group``, i.e. ``repeat_kv``),
    ``src/linattn/variants/selection.py:203-212``.  Returns float64
    ``(B,Hq,Tq,n_pages)``.
    """
    b, hq, tq, d = q.shape
    hkv = mins.shape[1]
    group = hq // hkv
    q64 = q.astype(np.float64)
    mn = np.repeat(mins.astype(np.float64), group, axis=1)  # (B,Hq,n,D)
    mx = np.repeat(maxs.astype(np.float64), group, axis=1)
    qe = q64[:, :, :, None, :]  # (B,Hq,Tq,1,D)
    return np.maximum(qe * mn[:, :, None], qe * mx[:, :, None]).sum(-1)


def topk_lowest_index(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the ``k`` largest entries of the last axis, sorted by descending
    score, ties broken by the LOWEST index.

    The reference uses ``torch.topk`` (``src/linattn/variants/selection.py:51-59``,
    ``src/linattn/kernels/triton/quest_pages.py:76-77``), which on CPU returns an
    arbitrary member of a tie; the build fixes the tie rule to lowest-index, which
    equals a stable descending sort.  On tie-free rows both agree exactly.
    """
    order = np.argsort(-scores, axis=-1, kind="stable")
    return order[..., :k].astype(np.int64)


def _masked_scores(q, mins, maxs, page_size, offset, sink_pages, n_pages_valid=None):
    """Scores with the visibility mask and the forced pages applied.

    ``quest_pages.py:67-75`` masks pages whose start lies after the query position to
    -inf and sets the query's own page to +inf.  The own-page scatter is taken
    per query row as in ``src/linattn/variants/selection.py:220-230`` (the operator
    at ``quest_pages.py:75`` writes every row's own page into every row when
    ``T_q > 1``; both agree at ``T_q == 1``).  ``sink_pages`` leading pages are also
    forced to +inf (the BASELINE's always-kept sink page).  ``n_pages_valid``
    (per batch) hides pages past a ragged sequence end.
    """
    scores = page_scores(q, mins, maxs)
    b, hq, tq, n = scores.shape
    q_pos = np.arange(tq) + offset
    page_start = np.arange(n) * page_size
    visible = page_start[None, :] <= q_pos[:, None]  # (Tq, n)
    visible = np.broadcast_to(visible, (b, tq, n)).copy()
    n_eff = np.full(b, n, dtype=np.int64) if n_pages_valid is None else np.asarray(n_pages_valid, np.int64)
    for bi in range(b):
        visible[bi, :, n_eff[bi]:] = False
    scores = np.where(visible[:, None], scores, -np.inf)
    for bi in range(b):
        own = np.minimum(q_pos // page_size, n_eff[bi] - 1)
        scores[bi, :, np.arange(tq), own] = np.inf
        for sp in range(min(sink_pages, n_eff[bi])):
            vis = visible[bi, :, sp]
            scores[bi, :, vis, sp] = np.inf
    return scores, n_eff


def page_select(q, mins, maxs, page_size: int, topk: int, *, offset: int = 0, sink_pages: int = 0,
                n_pages_valid=None):
    """Top-k page ids per query plus the masked page scores.

    ``src/linattn/kernels/triton/quest_pages.py:57-78`` with the per-row own page of
    ``selection.py:220-230``.  ``k = max(1, min(topk, n_pages))`` (``quest_pages.py:76``).
    Returns ``ids (B,Hq,Tq,k) int64`` and ``scores (B,Hq,Tq,n_pages) float64``.
    With ragged ``n_pages_valid`` the row of batch ``b`` keeps ``min(topk, n_b)``
    valid ids; the remaining slots are -1.
    """
    scores, n_eff = _masked_scores(q, mins, maxs, page_size, offset, sink_pages, n_pages_valid)
    n = scores.shape[-1]
    k = max(1, min(topk, n))
    ids = topk_lowest_index(scores, k)
    for bi in range(scores.shape[0]):
        kb = max(1, min(topk, int(n_eff[bi])))
        ids[bi, ..., kb:] = -1
    return ids, scores


def gqa_union(ids: np.ndarray, n_pages: int, group: int) -> np.ndarray:
    """Boolean page sets ``(B,Hkv,Tq,n_pages)``: the union over the query heads of a
    kv group (``src/linattn/variants/selection.py:232-235``)."""
    b, hq, tq, k = ids.shape
    sel = np.zeros((b, hq, tq, n_pages), dtype=bool)
    bi, hi, ti, ki = np.indices(ids.shape)
    valid = ids >= 0
    sel[bi[valid], hi[valid], ti[valid], ids[valid]] = True
    return sel.reshape(b, hq // group, group, tq, n_pages).any(axis=2)


def quest_effective_mask(q, k, page_size: int, topk: int, *, offset: int = 0, group: int = 1,
                         gqa_union_mode: bool = True, sink_pages: int = 0):
    """Token read mask of ``QuestAttention`` (``selection.py:86-108`` + ``:214-244``).

    Returns ``(B,Hq,Tq,Tk) bool``: selected pages (union over the group when
    ``gqa_union_mode``), expanded to tokens, intersected with causality, with the
    empty-row fallback to the diagonal.
    """
    tk = k.shape[2]
    mins, maxs = page_bounds(k, page_size)
    ids, _ = page_select(q, mins, maxs, page_size, topk, offset=offset, sink_pages=sink_pages)
    n = mins.shape[2]
    b, hq, tq, _ = ids.shape
    if gqa_union_mode and group > 1:
        sel = np.repeat(gqa_union(ids, n, group), group, axis=1)
    else:
        sel = gqa_union(ids, n, 1)
    tok = np.repeat(sel, page_size, axis=-1)[..., :tk]
    qpos = np.arange(tq) + offset
    causal = np.arange(tk)[None, :] <= qpos[:, None]
    allow = tok & causal
    empty = ~allow.any(-1)
    if empty.any():
        diag = np.minimum(qpos, tk - 1)
        for idx in zip(*np.nonzero(empty)):
            allow[idx + (diag[idx[-1]],)] = True
    return allow
