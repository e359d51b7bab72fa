"""Attention oracles: dense, block-sparse gather, paged sparse decode, (o, lse) merge.

Test infrastructure only (see ``oracle/__init__.py``).  All arithmetic in float64.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = ["dense_attention", "block_sparse_attention", "paged_sparse_decode", "lse_merge",
           "attention_with_lse"]


def _softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(x - m)
    return e / e.sum(-1, keepdims=True)


def dense_attention(q, k, v, *, causal: bool = True, scale=None, mask=None, offset=None):
    """Plain softmax attention with GQA (``src/linattn/core.py:148-181``).

    ``mask`` (broadcastable to ``(B,Hq,Tq,Tk)``) wins over ``causal``; with ``causal``
    and ``Tq != Tk`` the queries sit at the end (``core.py:168-170``) unless
    ``offset`` is given.
    """
    q64, k64, v64 = (x.astype(np.float64) for x in (q, k, v))
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    group = q.shape[1] // k.shape[1]
    kr = np.repeat(k64, group, axis=1)
    vr = np.repeat(v64, group, axis=1)
    s = np.einsum("bhtd,bhsd->bhts", q64, kr) * scale
    tq, tk = q.shape[2], k.shape[2]
    if mask is not None:
        allow = mask
    elif causal:
        off = (tk - tq) if offset is None else offset
        allow = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + off)
    else:
        allow = None
    if allow is not None:
        s = np.where(allow, s, -np.inf)
    return np.einsum("bhts,bhsd->bhtd", _softmax(s), vr)


def block_sparse_attention(q, k, v, block_ids, *, block_size: int):
    """Attention of each query over its kv head's selected key blocks.

    ``src/linattn/kernels/triton/block_sparse.py:40-75``: ``block_ids`` is
    ``(B,Hkv,N)`` (shared by all queries) or ``(B,Hkv,Tq,N)``; tokens at positions
    ``>= T_k`` are masked; no causal mask; duplicated ids count twice (the gather
    reads them twice); scale ``1/sqrt(D)``.  A row with no valid token returns 0
    (the reference's torch path returns NaN there, its Triton kernel 0).
    """
    b, hq, tq, d = q.shape
    hkv, tk = k.shape[1], k.shape[2]
    group = hq // hkv
    ids = np.asarray(block_ids, dtype=np.int64)
    if ids.ndim == 3:
        ids = np.broadcast_to(ids[:, :, None, :], (b, hkv, tq, ids.shape[-1]))
    out = np.zeros((b, hq, tq, d), dtype=np.float64)
    offs = np.arange(block_size)
    for bi in range(b):
        for kh in range(hkv):
            for t in range(tq):
                raw = (ids[bi, kh, t][:, None] * block_size + offs[None, :]).reshape(-1)
                valid = raw < tk
                pos = raw[valid]
                if pos.size == 0:
                    continue
                ks = k[bi, kh, pos].astype(np.float64)
                vs = v[bi, kh, pos].astype(np.float64)
                for g in range(group):
                    h = kh * group + g
                    s = ks @ q[bi, h, t].astype(np.float64) / math.sqrt(d)
                    p = _softmax(s)
                    out[bi, h, t] = p @ vs
    return out


def attention_with_lse(q_vec, ks, vs, scale):
    """``(o, lse)`` of one query over the rows ``ks``/``vs`` (float64); empty -> (0, -inf)."""
    if ks.shape[0] == 0:
        return np.zeros(q_vec.shape[-1]), -np.inf
    s = ks.astype(np.float64) @ q_vec.astype(np.float64) * scale
    m = s.max()
    e = np.exp(s - m)
    l = e.sum()
    return (e @ vs.astype(np.float64)) / l, m + math.log(l)


def paged_sparse_decode(q, k_pool, v_pool, page_table, seq_lens, lists, counts, *, page_size: int,
                        scale=None, k_scale=None, v_scale=None, q_pos=None, return_lse=False):
    """Decode attention over per-(batch, kv-head) page lists in a paged pool.

    The paged pool is the build's physical layout for the reference's logical cache
    (page ``p`` of ``(b, h)`` is ``K[b, h, p*P:(p+1)*P]``, ``quest_pages.py:38-48``):
    ``k_pool[page_table[b, p], h]`` holds those ``P`` rows.  ``lists[b, h, :counts[b,h]]``
    are logical page ids; all ``Hq/Hkv`` query heads of kv head ``h`` read them
    (the GQA union of ``selection.py:232-235``).  Rows at positions ``>= seq_lens[b]``
    or ``> q_pos[b]`` are masked.  ``k_scale``/``v_scale`` ``[N_phys, Hkv]`` dequantise
    fp8 codes given as float arrays.  ``q``: ``(B, Hq, D)``.  Returns ``(B, Hq, D)``
    (and ``lse (B, Hq)``).
    """
    b, hq, d = q.shape
    hkv = k_pool.shape[1]
    group = hq // hkv
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = np.zeros((b, hq, d))
    lse = np.full((b, hq), -np.inf)
    for bi in range(b):
        limit = int(seq_lens[bi]) if q_pos is None else min(int(seq_lens[bi]), int(q_pos[bi]) + 1)
        for kh in range(hkv):
            rows_k, rows_v = [], []
            for p in lists[bi, kh, : int(counts[bi, kh])]:
                p = int(p)
                phys = int(page_table[bi, p])
                nv = max(0, min(page_size, limit - p * page_size))
                if nv == 0:
                    continue
                kk = k_pool[phys, kh, :nv].astype(np.float64)
                vv = v_pool[phys, kh, :nv].astype(np.float64)
                if k_scale is not None:
                    kk = kk * float(k_scale[phys, kh])
                if v_scale is not None:
                    vv = vv * float(v_scale[phys, kh])
                rows_k.append(kk)
                rows_v.append(vv)
            ks = np.concatenate(rows_k) if rows_k else np.zeros((0, d))
            vs = np.concatenate(rows_v) if rows_v else np.zeros((0, d))
            for g in range(group):
                h = kh * group + g
                out[bi, h], lse[bi, h] = attention_with_lse(q[bi, h], ks, vs, scale)
    return (out, lse) if return_lse else out


def lse_merge(o_parts: np.ndarray, lse_parts: np.ndarray):
    """Merge split-KV partials: ``o = sum_i exp(lse_i - L) o_i``, ``L = logsumexp_i lse_i``.

    There is no reference function for this (the reference never splits the KV
    axis); it is the log-sum-exp identity, checked in the tests against dense
    attention over the union of the split ranges.  ``o_parts (S, ..., D)``,
    ``lse_parts (S, ...)``.  All-empty rows give ``o = 0, L = -inf``.
    """
    lse = lse_parts.astype(np.float64)
    m = lse.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lse - m_safe[None])
    tot = w.sum(axis=0)
    L = np.where(tot > 0, m_safe + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    o = (w[..., None] * o_parts.astype(np.float64)).sum(axis=0) / np.where(tot > 0, tot, 1.0)[..., None]
    return o, L
