"""CSA2 compressed sparse attention restated in numpy.  Test infrastructure only.

Follows ``CSA2Attention`` (``src/linattn/variants/csa2.py``):

* ``compressed_kv`` (:73-81): keys / values mean-pooled in groups of ``ratio`` tokens
  (``block_reduce``, ``src/linattn/core.py:103-120``, tail padded by repeating the
  last token) in the input dtype, then, for 4 or 8 bits, quantised group-wise along
  the channels and dequantised (``src/linattn/kv/quant.py:76-109``) and cast back to
  the input dtype;
* ``indexer_scores`` (:83-92): ``sum_e softmax(w)_e * ReLU(q_idx_e . k_idx_e)`` with
  ``q_idx = q @ q_proj[h]`` and ``k_idx = kc @ q_proj[h]`` (kc repeated to the query
  heads);
* ``attend`` (:95-140): a group is eligible when it ends at or before the query and
  before the raw window ``[p - w + 1, p]`` (``w = max(1, min(window, T_k))``); the top
  ``max(1, min(topk_groups, n_groups))`` scores, intersected with eligibility, plus the
  window are attended in ONE softmax over the raw keys followed by the pooled ones.

Rounding follows what the reference computes on the CPU: the pooled mean is the
float32 sum of the ``ratio`` rows divided by ``ratio`` and rounded once to the input
dtype (torch's CPU ``mean`` of bf16 / f16 rounds once); the codec works in float32
(true divisions, FP4 nearest grid magnitude with the first index on ties, FP8 round to
nearest even); the dequantised value is rounded once to the input dtype.  The indexer
and the attention run in float64.
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np

from oracle.attention import _softmax
from oracle.quant import e4m3_decode, e4m3_encode
from oracle.quest import topk_lowest_index

__all__ = ["FP4_GRID", "round_to_dtype", "pool_mean", "quant_roundtrip", "compressed_kv", "csa2_scores",
           "csa2_select", "csa2_attend", "csa2_forward", "boundary_tied_rows"]

# E2M1 magnitudes (src/linattn/kv/quant.py:36); codes 8..15 carry the sign
FP4_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> the nearest value of ``dtype`` ('bf16', 'f16' or 'f32'), ties to even,
    returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(dtype)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def pool_mean(x: np.ndarray, ratio: int, dtype: str) -> np.ndarray:
    """``block_reduce(x, ratio, -2)`` (``src/linattn/core.py:103-120``) on (..., T, D)
    values of ``dtype``: float32 sum of each group's rows in order, divided by
    ``ratio``, rounded once to ``dtype``."""
    x = np.asarray(x, dtype=np.float32)
    if ratio == 1:
        return x.copy()
    t = x.shape[-2]
    n_groups = -(-t // ratio)
    acc = np.zeros((*x.shape[:-2], n_groups, x.shape[-1]), dtype=np.float32)
    for i in range(ratio):
        rows = np.minimum(np.arange(n_groups) * ratio + i, t - 1)  # tail repeats the last row
        acc = (acc + x[..., rows, :]).astype(np.float32)
    return round_to_dtype(acc / np.float32(ratio), dtype)


def quant_roundtrip(x: np.ndarray, bits: int, group: int = 32) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``dequantize(*quantize(x))`` (``src/linattn/kv/quant.py:76-109``) in float32 along
    the last axis, tail groups zero-padded.  Returns ``(x_hat, codes, scales)``: codes
    int8 FP4 indices (0..15) or uint8 e4m3 bytes, scales (..., n_groups)."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    pad = (-d) % group
    xp = np.concatenate([x, np.zeros((*x.shape[:-1], pad), np.float32)], axis=-1) if pad else x
    g = xp.reshape(*xp.shape[:-1], -1, group)
    amax = np.abs(g).max(-1, keepdims=True)
    top = np.float32(6.0) if bits == 4 else np.float32(448.0)
    scale = (np.maximum(amax, np.float32(1e-8)) / top).astype(np.float32)
    n = (g / scale).astype(np.float32)
    if bits == 4:
        dist = np.abs(np.abs(n)[..., None] - FP4_GRID)
        idx = dist.argmin(-1)  # first index on ties
        mag = FP4_GRID[idx]
        value = np.where(n < 0, -mag, mag).astype(np.float32)
        codes = np.where(n < 0, idx + 8, idx).astype(np.int8)
    elif bits == 8:
        codes = e4m3_encode(n)
        value = e4m3_decode(codes)
    else:
        raise ValueError("bits must be 4 or 8")
    x_hat = (value * scale).astype(np.float32).reshape(*xp.shape[:-1], -1)[..., :d]
    return x_hat, codes.reshape(*xp.shape[:-1], -1)[..., :d], scale[..., 0]


def compressed_kv(x: np.ndarray, ratio: int, bits: int, group: int, dtype: str) -> np.ndarray:
    """``CSA2Attention.compressed_kv`` for one of k / v (``csa2.py:73-81``): float32
    array holding ``dtype`` values."""
    pooled = pool_mean(x, ratio, dtype)
    if bits >= 16:
        return pooled
    return round_to_dtype(quant_roundtrip(pooled, bits, group)[0], dtype)


def csa2_scores(q, kc, q_proj, head_weights) -> np.ndarray:
    """``CSA2Attention.indexer_scores`` (``csa2.py:83-92``), float64 ``(B, Hq, Tq, G)``."""
    b, hq, tq, d = q.shape
    group = hq // kc.shape[1]
    kr = np.repeat(kc.astype(np.float64), group, axis=1)
    proj = q_proj.astype(np.float64)
    q_idx = np.einsum("bhtd,hedf->bhtef", q.astype(np.float64), proj)
    k_idx = np.einsum("bhsd,hedf->bhsef", kr, proj)
    dots = np.einsum("bhtef,bhsef->bhtse", q_idx, k_idx)
    w = np.exp(head_weights.astype(np.float64) - np.max(head_weights))
    w = w / w.sum()
    return (np.maximum(dots, 0.0) * w).sum(-1)


def _eligible(n_groups: int, ratio: int, t_q: int, offset: int, w: int) -> np.ndarray:
    """(T_q, G): group g ends at or before the query and before its window
    (``csa2.py:107-112``)."""
    q_pos = np.arange(t_q)[:, None] + offset
    end = (np.arange(n_groups)[None, :] + 1) * ratio - 1
    return (end <= q_pos) & (end < q_pos - w + 1)


def csa2_select(scores: np.ndarray, ratio: int, window: int, topk_groups: int, t_k: int,
                offset: int = 0) -> np.ndarray:
    """Selected groups (``csa2.py:113-120``) as a bool ``(B, Hq, Tq, G)`` mask: top
    ``max(1, min(topk_groups, G))`` of the eligible scores (lowest index on ties),
    intersected with eligibility."""
    b, h, t_q, n_groups = scores.shape
    w = max(1, min(window, t_k))
    elig = _eligible(n_groups, ratio, t_q, offset, w)
    s = np.where(elig, scores, -np.inf)
    keep = max(1, min(topk_groups, n_groups))
    idx = topk_lowest_index(s, keep)
    mask = np.zeros(scores.shape, dtype=bool)
    np.put_along_axis(mask, idx, True, axis=-1)
    return mask & elig


def csa2_attend(q, k, v, q_proj, head_weights, *, ratio: int, bits: int, group: int, window: int,
                topk_groups: int, offset: int = 0, dtype: str = "f32") -> Tuple[np.ndarray, Dict[str, float]]:
    """``CSA2Attention.attend`` (``csa2.py:95-140``) for queries at ``offset ..`` over
    the cached ``k, v (B, Hkv, T_k, D)``.  Returns ``(out float64, stats)``."""
    t_q, t_k = q.shape[2], k.shape[2]
    kc = compressed_kv(k, ratio, bits, group, dtype)
    vc = compressed_kv(v, ratio, bits, group, dtype)
    scores = csa2_scores(q, kc, q_proj, head_weights)
    gmask = csa2_select(scores, ratio, window, topk_groups, t_k, offset)
    w = max(1, min(window, t_k))
    q_pos = np.arange(t_q)[:, None] + offset
    kj = np.arange(t_k)[None, :]
    wmask = np.broadcast_to((kj <= q_pos) & (q_pos - kj < w), (*q.shape[:2], t_q, t_k))
    allow = np.concatenate([wmask, gmask], axis=-1)
    k_all = np.concatenate([k.astype(np.float64), kc.astype(np.float64)], axis=2)
    v_all = np.concatenate([v.astype(np.float64), vc.astype(np.float64)], axis=2)
    rep = q.shape[1] // k.shape[1]
    kr, vr = np.repeat(k_all, rep, axis=1), np.repeat(v_all, rep, axis=1)
    s = np.einsum("bhtd,bhsd->bhts", q.astype(np.float64), kr) / math.sqrt(q.shape[-1])
    out = np.einsum("bhts,bhsd->bhtd", _softmax(np.where(allow, s, -np.inf)), vr)
    groups = float(gmask.sum(-1).mean())
    window_reads = float(wmask.sum(-1).mean())
    stats = {"groups_per_query": groups, "tokens_equivalent": groups * ratio + window_reads, "bits": float(bits),
             "reads_per_query": groups + window_reads}
    return out, stats


def csa2_forward(q, k, v, q_proj, head_weights, *, chunk: int, **kw) -> Tuple[np.ndarray, Dict[str, float]]:
    """The reference's chunked forward (``src/linattn/core.py:231-271``): chunk ``c``
    attends its queries at offset ``start`` over the keys up to its end.  The stats
    are the last chunk's."""
    t = q.shape[2]
    outs, stats = [], {}
    for start in range(0, t, chunk):
        stop = min(start + chunk, t)
        o, stats = csa2_attend(q[:, :, start:stop], k[:, :, :stop], v[:, :, :stop], q_proj, head_weights,
                               offset=start, **kw)
        outs.append(o)
    return np.concatenate(outs, axis=2), stats


def boundary_tied_rows(scores: np.ndarray, *, ratio: int, window: int, topk_groups: int, chunk: int,
                       rel: float = 1e-6) -> np.ndarray:
    """(H, T) bool for scores (H, T, G) of one sequence: rows whose selection is decided
    by a tie (the last kept and the first dropped eligible scores within ``rel``), where
    the reference's top-k order and this library's lowest-index rule may pick different
    groups.  Queries are at positions 0..T-1, attended in chunks of ``chunk``."""
    h, t, n_groups = scores.shape
    keep = max(1, min(topk_groups, n_groups))
    tied = np.zeros((h, t), dtype=bool)
    for tt in range(t):
        t_k = min(t, (tt // chunk + 1) * chunk)
        w = max(1, min(window, t_k))
        elig = (np.arange(n_groups) + 1) * ratio <= tt - w + 1
        if elig.sum() <= keep:
            continue
        for hh in range(h):
            srt = np.sort(scores[hh, tt][elig])[::-1]
            tied[hh, tt] = abs(srt[keep - 1] - srt[keep]) <= rel * max(1.0, abs(srt[keep]))
    return tied
