"""Block-granular selectors for prefill (MInference block-sparse, MoBA, the sink +
window + top-k composition).  numpy restatement; test infrastructure only."""

from __future__ import annotations

import math

import numpy as np

from oracle.quest import topk_lowest_index

__all__ = ["block_reduce", "minference_block_select", "moba_select", "window_block_select",
           "block_mask_to_token_mask"]


def block_reduce(x: np.ndarray, block: int, axis: int = -2) -> np.ndarray:
    """Mean-pool along ``axis`` in blocks of ``block``; the tail is padded by
    repeating the last row (``src/linattn/core.py:103-120``)."""
    if block == 1:
        return x.astype(np.float64)
    x = np.moveaxis(x.astype(np.float64), axis, -2)
    t = x.shape[-2]
    pad = (-t) % block
    if pad:
        x = np.concatenate([x, np.repeat(x[..., -1:, :], pad, axis=-2)], axis=-2)
    x = x.reshape(*x.shape[:-2], x.shape[-2] // block, block, x.shape[-1]).mean(axis=-2)
    return np.moveaxis(x, -2, axis)


def block_mask_to_token_mask(sel, block_q: int, block_k: int, t_q: int, t_k: int):
    """``src/linattn/variants/selection.py:45-48``."""
    return np.repeat(np.repeat(sel, block_q, axis=-2), block_k, axis=-1)[..., :t_q, :t_k]


def _topk_mask(scores, k, allowed):
    """``topk_blocks`` (``selection.py:51-59``) with lowest-index ties."""
    s = np.where(allowed, scores, -np.inf)
    kk = max(1, min(k, s.shape[-1]))
    idx = topk_lowest_index(s, kk)
    out = np.zeros(s.shape, dtype=bool)
    np.put_along_axis(out, idx, True, axis=-1)
    return out


def pooled_block_scores(q, k, block: int):
    """``mean(q_blk) . mean(k_blk) / sqrt(D)`` per (b, q-head, q-block, k-block) with
    GQA repeat (``selection.py:343-346``)."""
    group = q.shape[1] // k.shape[1]
    qp = block_reduce(q, block, -2)
    kp = block_reduce(np.repeat(k, group, axis=1), block, -2)
    return np.einsum("bhqd,bhkd->bhqk", qp, kp) / math.sqrt(q.shape[-1])


def minference_block_select(q, k, block: int, topk: int, *, offset: int = 0, sink_size: int = 0):
    """Token mask of ``MInferenceAttention._block_sparse`` (``selection.py:339-353``):
    causal block top-k on pooled scores, plus the own (diagonal) block, plus the first
    ``sink_size`` tokens.  Not intersected with token causality (``effective_mask``
    does that, ``selection.py:96-99``)."""
    t_q, t_k = q.shape[-2], k.shape[-2]
    scores = pooled_block_scores(q, k, block)
    n_qb, n_kb = scores.shape[-2:]
    qb = (np.arange(n_qb) + offset // block)[:, None]
    kb = np.arange(n_kb)[None, :]
    sel = _topk_mask(scores, topk, kb <= qb) | (kb == qb)
    mask = block_mask_to_token_mask(sel, block, block, t_q, t_k)
    return mask | (np.arange(t_k)[None, :] < sink_size)


def moba_select(q, k, block: int, topk: int, *, offset: int = 0):
    """Token mask of ``MoBAAttention.select`` (``selection.py:635-649``): per-token
    gate ``q . mean(k_blk) / sqrt(D)``, causal block top-k, plus the own block."""
    t_q, t_k = q.shape[-2], k.shape[-2]
    group = q.shape[1] // k.shape[1]
    n_kb = (t_k + block - 1) // block
    kp = block_reduce(np.repeat(k, group, axis=1), block, -2)
    gates = np.einsum("bhtd,bhkd->bhtk", q.astype(np.float64), kp) / math.sqrt(q.shape[-1])
    q_pos = np.arange(t_q) + offset
    allowed = (np.arange(n_kb) * block)[None, :] <= q_pos[:, None]
    sel = _topk_mask(gates, topk, allowed)
    own = np.minimum(q_pos // block, n_kb - 1)
    sel[..., np.arange(t_q), own] = True
    return block_mask_to_token_mask(sel, 1, block, t_q, t_k)


def window_block_select(q, k, block: int, topk: int, *, window_blocks: int, sink_blocks: int = 1):
    """Block lists of the BASELINE's block-sparse prefill (config 4): per (b, q-head,
    q-block ``i``) the sink blocks ``[0, sink_blocks)``, the window ``[i-window_blocks+1, i]``
    and the ``topk`` highest pooled-score blocks among the remaining causal blocks
    ``kb < i``.  Same pooled score as ``selection.py:343-346``; lowest-index ties.

    Returns ``(ids (B,Hq,n_qb,n_max) int64 ascending, -1 padded; counts (B,Hq,n_qb))``.
    """
    scores = pooled_block_scores(q, k, block)
    b, hq, n_qb, n_kb = scores.shape
    kb = np.arange(n_kb)[None, :]
    qb = np.arange(n_qb)[:, None]
    forced = (kb < sink_blocks) | ((kb <= qb) & (kb > qb - window_blocks))
    forced &= kb <= qb
    cand = (kb <= qb) & ~forced
    s = np.where(cand, scores, -np.inf)
    kk = max(1, min(topk, n_kb))
    idx = topk_lowest_index(s, kk)
    vals = np.take_along_axis(s, idx, axis=-1)
    sel = np.broadcast_to(forced, scores.shape).copy()
    bi, hi, qi, ki = np.indices(idx.shape)
    ok = np.isfinite(vals)
    sel[bi[ok], hi[ok], qi[ok], idx[ok]] = True
    counts = sel.sum(-1)
    n_max = int(counts.max())
    ids = np.full((b, hq, n_qb, n_max), -1, dtype=np.int64)
    for pos in np.ndindex(b, hq, n_qb):
        nz = np.nonzero(sel[pos])[0]
        ids[pos][: nz.size] = nz
    return ids, counts
