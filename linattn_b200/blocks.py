"""Block selection for block-sparse attention on the B200.

* ``block_mean``: mean-pooled blocks of queries / keys (``block_reduce``,
  ``src/linattn/core.py:103-120``), a CUDA kernel.
* ``block_score_topk``: one kernel for the rest of every block selector: the fp32
  block scores of each row against its kv head's candidates, the causal top-k
  (lowest-index ties) and the ascending merge with the forced blocks, never writing
  the score matrix (``linattn_block_score_topk``).
* ``pooled_block_scores``: ``mean(q_blk) . mean(k_blk) / sqrt(D)`` per (b, q-head,
  q-block, k-block) (``MInferenceAttention._block_sparse``,
  ``src/linattn/variants/selection.py:339-347``) as a full matrix, from the same kernel
  (for inspection and tests; the selection itself does not materialise it).
* ``block_select``: per q-block lists = the top-k causal candidate blocks united with
  forced blocks: the own block (MInference, ``selection.py:350-351``) and/or sink
  blocks and a window of blocks (the block-sparse prefill's sink + window + top-k).
* ``moba_select``: per-token lists of ``MoBAAttention.select`` (``selection.py:635-649``):
  gate ``q . mean(k_blk) / sqrt(D)``, top-k over blocks that start at or before the
  query, plus the own block.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple, Union

import torch

from linattn_b200 import _lib as L

__all__ = ["block_mean", "block_score_topk", "pooled_block_scores", "block_select", "moba_select", "merge_block_lists",
           "block_sparse_prefill"]


def block_mean(x: torch.Tensor, block: int) -> torch.Tensor:
    """``(B,H,T,D)`` -> ``(B,H,ceil(T/block),D)`` fp32 block means (tail repeats the last row)."""
    L.require_cuda(x)
    b, h, t, d = x.shape
    nb = -(-t // block)
    out = torch.empty(b, h, nb, d, dtype=torch.float32, device=x.device)
    L.check(L.lib().linattn_block_mean(x.data_ptr(), L.dtype_code(x), b, h, t, d, L.strides4(x), block,
                                       out.data_ptr(), L.stream_of(x)))
    return out


def block_score_topk(a: torch.Tensor, bm: torch.Tensor, k: int, *, scale: float, first_pos: int, key_block: int = 1,
                     skip: int = 0, merge_pos: int, own_div: int = 1, sink: int = 0, window: int = 0,
                     force_own: bool = True, n_max: int = 0, topk_out: bool = False,
                     scores_out: Optional[torch.Tensor] = None):
    """Rows ``a (B, H_q, R, D)`` against candidates ``bm (B, H_kv, NC, D)`` (see
    ``linattn_block_score_topk``): returns ``(ids (B, H_q, R, n_max) int32 ascending,
    -1 padded, counts (B, H_q, R) int32)`` and, with ``topk_out``, the top k in score
    order ``(B, H_q, R, k)``.  ``scores_out`` (B, H_q, R, NC) fp32, if given, receives
    the scores the selection ranked (other entries untouched)."""
    L.require_cuda(a, bm)
    b, hq, r, d = a.shape
    hkv, nc = bm.shape[1], bm.shape[2]
    kk = max(1, min(int(k), nc))
    n_max = n_max or (kk + max(sink, 0) + max(window, 1))
    out = torch.empty(b, hq, r, n_max, dtype=torch.int32, device=a.device)
    counts = torch.empty(b, hq, r, dtype=torch.int32, device=a.device)
    tk = torch.empty(b, hq, r, kk, dtype=torch.int32, device=a.device) if topk_out else None
    if scores_out is not None and (scores_out.shape != (b, hq, r, nc) or scores_out.dtype != torch.float32
                                   or not scores_out.is_contiguous()):
        raise ValueError("scores_out must be a contiguous fp32 (B, H_q, R, NC) tensor")
    L.check(L.lib().linattn_block_score_topk(
        a.data_ptr(), L.dtype_code(a), L.strides4(a), bm.data_ptr(), L.dtype_code(bm), L.strides4(bm), b, hq, hkv, r,
        nc, d, float(scale), kk, first_pos, key_block, skip, merge_pos, own_div, sink, window, int(force_own),
        out.data_ptr(), n_max, counts.data_ptr(), L.ptr(tk), L.ptr(scores_out), L.stream_of(a)))
    return (out, counts, tk) if topk_out else (out, counts)


def pooled_block_scores(q: torch.Tensor, k: torch.Tensor, block: int) -> torch.Tensor:
    """``(B,H_q,n_qb,n_kb)`` fp32 pooled block scores with the GQA repeat of ``k``: the
    scores ``block_select`` ranks (computed by the same kernel; entries past a row's
    own block are -inf)."""
    b, hq, _, d = q.shape
    qp, kp = block_mean(q, block), block_mean(k, block)
    nqb, nkb = qp.shape[2], kp.shape[2]
    s = torch.full((b, hq, nqb, nkb), float("-inf"), dtype=torch.float32, device=q.device)
    block_score_topk(qp, kp, 1, scale=1.0 / math.sqrt(d), first_pos=0, merge_pos=0, scores_out=s)
    return s


def merge_block_lists(topk_ids: torch.Tensor, *, period: int, first_pos: int, own_div: int, n_blocks: int,
                      sink: int = 0, window: int = 0, force_own: bool = True,
                      n_max: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Ascending union of ``topk_ids (..., k)`` with the forced blocks (see
    ``linattn_merge_block_lists``); returns ``(ids (..., n_max) int32, counts (...) int32)``."""
    k = topk_ids.shape[-1]
    rows = topk_ids.numel() // max(k, 1)
    n_max = n_max or (k + sink + max(window, 1))
    out = torch.empty(*topk_ids.shape[:-1], n_max, dtype=torch.int32, device=topk_ids.device)
    counts = torch.empty(topk_ids.shape[:-1], dtype=torch.int32, device=topk_ids.device)
    tk = topk_ids.to(torch.int32).contiguous()
    L.check(L.lib().linattn_merge_block_lists(tk.data_ptr(), rows, k, period, first_pos, own_div, n_blocks, sink,
                                              window, int(force_own), out.data_ptr(), n_max, counts.data_ptr(),
                                              L.stream_of(tk)))
    return out, counts


def block_select(q: torch.Tensor, k: torch.Tensor, block: int, topk: int, *, offset: int = 0, sink_blocks: int = 0,
                 window_blocks: int = 0, force_own: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per (b, q-head, q-block) block lists, ascending, -1 padded, with counts.

    Candidates of q-block ``i`` (absolute block ``qb = offset // block + i``): blocks
    ``[sink_blocks, qb - window_blocks]`` (``kb <= qb`` when ``window_blocks == 0``); the
    top ``topk`` of their pooled scores are united with ``[0, sink_blocks)``, the window
    ``[qb - window_blocks + 1, qb]`` and, with ``force_own``, ``qb``.
    ``window_blocks = sink_blocks = 0, force_own`` is MInference's block-sparse pattern."""
    b, hq, _, d = q.shape
    qp, kp = block_mean(q, block), block_mean(k, block)
    qb0 = offset // block
    kk = max(1, min(topk, kp.shape[2]))
    # causal candidates of row i: [sink_blocks, qb0 + i - window_blocks]
    return block_score_topk(qp, kp, kk, scale=1.0 / math.sqrt(d), first_pos=qb0 - window_blocks, key_block=1,
                            skip=sink_blocks, merge_pos=qb0, own_div=1, sink=sink_blocks, window=window_blocks,
                            force_own=force_own, n_max=kk + sink_blocks + max(window_blocks, 1))


def moba_select(q: torch.Tensor, k: torch.Tensor, block: int, topk: int, *,
                offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per (b, q-head, query) block lists of MoBA (``selection.py:635-649``)."""
    b, hq, tq, d = q.shape
    kp = block_mean(k, block)
    kk = max(1, min(topk, kp.shape[2]))
    # a query never routes to a block that starts after it: block j visible iff j * block <= pos
    return block_score_topk(q, kp, kk, scale=1.0 / math.sqrt(d), first_pos=offset, key_block=block,
                            merge_pos=offset, own_div=block, force_own=True, n_max=kk + 1)


def block_sparse_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ids: torch.Tensor, *,
                         counts: Optional[torch.Tensor] = None, rows_per_list: int = 64, sink: int = 0,
                         causal: Union[bool, int] = True, window: int = 0, offset: int = 0,
                         scale: Optional[float] = None,
                         lse_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                         v_f16: Optional[bool] = None) -> torch.Tensor:
    """Block-sparse causal prefill on the tcgen05 tensor cores: query ``t`` reads the
    64-token key blocks of ``ids[b, h, t // rows_per_list]`` (ascending, -1 padded) plus
    the tokens below ``sink``.  ``q (B,H_q,T_q,128)``, ``k, v (B,H_kv,T_k,128)``, bf16 or f16.
    ``causal``: ``True`` / 1 reads keys ``<= offset + t``; an integer ``c > 1`` treats the
    keys as pooled groups of ``c`` tokens and reads key ``j`` once ``j * c <= offset + t
    + c - 1`` (NSA's compression branch).  ``window > 0`` (no sink): a query also skips the
    keys below ``offset + t - window + 1`` (a token-exact sliding window).

    For bf16 inputs, ``v_f16`` (default on) first copies V to f16 (exact up to a
    per-(b, kv head) power-of-two scale) so that the P V product takes one f16 P part
    instead of bf16 hi + lo parts."""
    dev = L.require_cuda(q, k, v, ids, counts, lse_out)
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise ValueError("q, k and v must have one dtype (bf16 or f16)")
    b, hq, tq, d = q.shape
    hkv, tk = k.shape[1], k.shape[2]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if ids.dtype != torch.int32 or ids.stride(-1) != 1:
        ids = ids.to(torch.int32).contiguous()
    if ids.dim() != 4:
        raise ValueError("ids must be (B, H_q, list rows, n)")
    cs = None
    if counts is not None:
        counts = counts.to(torch.int32)
        cs = (L.c_i64 * 3)(*counts.stride())
    if out is None:
        out = torch.empty_like(q)
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    status = L.status_word(dev)
    v16 = vsc = None
    if q.dtype == torch.bfloat16 and v_f16 is not False:
        v16 = torch.empty(v.shape, dtype=torch.float16, device=dev)
        vsc = torch.empty(b * hkv, dtype=torch.float32, device=dev)
        amax = torch.empty(b * hkv, dtype=torch.int32, device=dev)
        L.check(L.lib().linattn_prefill_v_to_f16(v.data_ptr(), b * hkv, tk * d, v16.data_ptr(), vsc.data_ptr(),
                                                 amax.data_ptr(), L.stream_of(q)))
    L.check(L.lib().linattn_block_sparse_prefill(
        q.data_ptr(), L.dtype_code(q), b, hq, tq, k.data_ptr(), v.data_ptr(), hkv, tk, d, ids.data_ptr(),
        L.ptr(counts), (L.c_i64 * 3)(*ids.stride()[:3]), ids.shape[-1], rows_per_list, cs, sink, int(causal),
        int(window), offset,
        scale, out.data_ptr(), L.strides4(out), L.ptr(lse_out), L.ptr(v16), L.ptr(vsc), status.data_ptr(),
        L.stream_of(q)))
    if L.strict():
        L.check_status(dev)
    return out
