"""Lightning-indexer scores and top-k (numpy restatement).  Test infrastructure only."""

from __future__ import annotations

import numpy as np

from oracle.quest import topk_lowest_index

__all__ = ["indexer_scores", "indexer_topk"]


def indexer_scores(q_idx, k_idx, head_weights, *, k_scale=None, group: int = 64) -> np.ndarray:
    """``I[b,t,s] = sum_h w[b,t,h] * ReLU(q_idx[b,t,h,:] . k_idx[b,s,h,:])``.

    ``src/linattn/kernels/triton/fused_indexer.py:52-60``.  ``k_scale (B, ceil(Tk/group))``
    dequantises fp8 key codes given as floats with one scale per ``group`` tokens
    (the BASELINE's per-64-token scales; the codec is ``src/linattn/kv/quant.py:90-109``
    applied along the token axis).  float64 ``(B,Tq,Tk)``.
    """
    k64 = k_idx.astype(np.float64)
    if k_scale is not None:
        tok_scale = np.repeat(np.asarray(k_scale, np.float64), group, axis=1)[:, : k_idx.shape[1]]
        k64 = k64 * tok_scale[:, :, None, None]
    dots = np.einsum("bqhd,bkhd->bqkh", q_idx.astype(np.float64), k64)
    return (np.maximum(dots, 0.0) * head_weights.astype(np.float64)[:, :, None, :]).sum(-1)


def indexer_topk(q_idx, k_idx, head_weights, k: int, *, causal: bool = False, offset: int = 0,
                 k_scale=None, group: int = 64):
    """Top-k indexer scores: ``fused_indexer.py:63-73`` (``k = min(k, T_k)``), values
    sorted descending with lowest-index ties.

    ``causal=True`` is the BASELINE's causal variant: keys after the query position
    (``s > offset + t``) are masked to -inf before the top-k; slots beyond the
    visible count hold value -inf and index -1.
    """
    s = indexer_scores(q_idx, k_idx, head_weights, k_scale=k_scale, group=group)
    tq, tk = s.shape[1], s.shape[2]
    kk = min(k, tk)
    if causal:
        allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + offset)
        s = np.where(allow[None], s, -np.inf)
    idx = topk_lowest_index(s, kk)
    vals = np.take_along_axis(s, idx, axis=-1)
    if causal:
        idx = np.where(np.isneginf(vals), -1, idx)
    return vals, idx
