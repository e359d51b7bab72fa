"""NSA three-branch attention restated in numpy.  Test infrastructure only.

Follows ``NSAAttention`` (``src/linattn/variants/native_sparse.py``):

* compression branch (:67-76): attention over the keys / values mean-pooled in groups of
  ``c = compress_ratio`` (``block_reduce`` in the input dtype), a query at ``p`` reading
  the groups that start at or before ``p + c - 1``;
* selection branch (:78-98): blocks of ``block_size`` raw tokens scored by
  ``q . mean(k over the block) / sqrt(D)`` (per query head), the top ``selected_blocks``
  of the blocks that start at or before ``p``, plus the query's own block; the
  selected blocks are read WHOLE (no causal cut inside the own block);
* window branch (:100-105): the ``window_size`` tokens ending at ``p``;
* combination (:107-119): per-head gates, uniform (1/3 each) or
  ``sigmoid(gates)`` normalised to sum 1.

One deliberate difference: when fewer than ``selected_blocks`` blocks start at or
before ``p``, the reference's ``topk_blocks`` fills the remainder with blocks that
start after ``p`` (torch's top-k picks among the -inf scores in an unspecified order);
here such a row reads its allowed blocks only.  Ties in the scores go to the lowest
block index.  Arithmetic in float64 (pooled means rounded to the input dtype first).
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import numpy as np

from oracle.attention import _softmax
from oracle.csa2 import pool_mean
from oracle.quest import topk_lowest_index

__all__ = ["nsa_block_scores", "nsa_select", "nsa_branches", "nsa_attend", "nsa_forward", "nsa_fill_rows"]


def _attend(q, k, v, allow):
    """Masked softmax attention with the GQA repeat, float64 (rows with nothing to read: 0)."""
    rep = q.shape[1] // k.shape[1]
    kr = np.repeat(k.astype(np.float64), rep, axis=1)
    vr = np.repeat(v.astype(np.float64), rep, axis=1)
    s = np.einsum("bhtd,bhsd->bhts", q.astype(np.float64), kr) / math.sqrt(q.shape[-1])
    p = _softmax(np.where(allow, s, -np.inf))
    return np.einsum("bhts,bhsd->bhtd", np.nan_to_num(p), vr)


def nsa_block_scores(q, k, block: int, dtype: str = "f32") -> np.ndarray:
    """``(B, Hq, Tq, n_kb)`` float64: ``q . block_reduce(repeat_kv(k), block) / sqrt(D)``
    (``native_sparse.py:81-84``)."""
    kp = pool_mean(k, block, dtype).astype(np.float64)
    kr = np.repeat(kp, q.shape[1] // k.shape[1], axis=1)
    return np.einsum("bhtd,bhsd->bhts", q.astype(np.float64), kr) / math.sqrt(q.shape[-1])


def nsa_select(scores: np.ndarray, block: int, selected: int, offset: int = 0) -> np.ndarray:
    """Selected blocks ``(B, Hq, Tq, n_kb)`` bool (``native_sparse.py:85-92``): top
    ``max(1, min(selected, n_kb))`` of the blocks starting at or before the query
    (lowest index on ties, no fill from later blocks), plus the own block
    ``min(p // block, n_kb - 1)``."""
    b, h, t_q, n_kb = scores.shape
    pos = np.arange(t_q) + offset
    allowed = (np.arange(n_kb)[None, :] * block) <= pos[:, None]
    kk = max(1, min(selected, n_kb))
    s = np.where(allowed, scores, -np.inf)
    idx = topk_lowest_index(s, kk)
    sel = np.zeros(scores.shape, dtype=bool)
    np.put_along_axis(sel, idx, True, axis=-1)
    sel &= allowed
    own = np.minimum(pos // block, n_kb - 1)
    sel[..., np.arange(t_q), own] = True
    return sel


def nsa_fill_rows(t_q: int, block: int, selected: int, n_kb: int, offset: int = 0) -> np.ndarray:
    """(Tq,) bool: queries with fewer allowed blocks than the reference's top-k size,
    where the reference reads torch-chosen later blocks."""
    pos = np.arange(t_q) + offset
    return (pos // block + 1) < max(1, min(selected, n_kb))


def nsa_branches(q, k, v, *, compress: int, block: int, selected: int, window: int, offset: int = 0,
                 dtype: str = "f32") -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """``(o_cmp, o_slc, o_win, sel)`` for queries at ``offset ..`` over the cached k, v."""
    b, hq, t_q, _ = q.shape
    t_k = k.shape[2]
    pos = (np.arange(t_q) + offset)[:, None]
    kc, vc = pool_mean(k, compress, dtype), pool_mean(v, compress, dtype)
    n_groups = kc.shape[2]
    allow_c = (np.arange(n_groups)[None, :] * compress) <= pos + compress - 1
    if not allow_c.any():
        allow_c = np.ones_like(allow_c)
    o_cmp = _attend(q, kc, vc, np.broadcast_to(allow_c, (b, hq, t_q, n_groups)))
    sel = nsa_select(nsa_block_scores(q, k, block, dtype), block, selected, offset)
    tok = np.repeat(sel, block, axis=-1)[..., :t_k]
    o_slc = _attend(q, k, v, tok)
    kj = np.arange(t_k)[None, :]
    allow_w = (kj <= pos) & ((pos - kj) < window)
    o_win = _attend(q, k, v, np.broadcast_to(allow_w, (b, hq, t_q, t_k)))
    return o_cmp, o_slc, o_win, sel


def nsa_attend(q, k, v, gates: Optional[np.ndarray] = None, **kw) -> Tuple[np.ndarray, Dict[str, float]]:
    """``NSAAttention.attend`` (``native_sparse.py:107-119``); ``gates`` (Hq, 3) raw
    parameters for the learned mode, ``None`` for uniform."""
    o_cmp, o_slc, o_win, sel = nsa_branches(q, k, v, **kw)
    if gates is None:
        g = np.full((q.shape[1], 3), 1.0 / 3.0)
    else:
        g = 1.0 / (1.0 + np.exp(-gates.astype(np.float64)))
        g = g / np.maximum(g.sum(-1, keepdims=True), 1e-9)
    out = (g[:, 0].reshape(1, -1, 1, 1) * o_cmp + g[:, 1].reshape(1, -1, 1, 1) * o_slc
           + g[:, 2].reshape(1, -1, 1, 1) * o_win)
    return out, {"selected_blocks_per_query": float(sel.sum(-1).mean())}


def nsa_forward(q, k, v, *, chunk: int, gates: Optional[np.ndarray] = None, **kw):
    """Chunked forward (``src/linattn/core.py:231-271``); stats of the last chunk."""
    t = q.shape[2]
    outs, stats = [], {}
    for start in range(0, t, chunk):
        stop = min(start + chunk, t)
        o, stats = nsa_attend(q[:, :, start:stop], k[:, :, :stop], v[:, :, :stop], gates, offset=start, **kw)
        outs.append(o)
    return np.concatenate(outs, axis=2), stats
