"""Token-sparse attention for DSA / CSA on the B200.

``token_sparse_attention`` runs the ``linattn_token_attention`` kernel: every query
attends to the union of its list's tokens (each list entry standing for ``block``
consecutive tokens), the first ``sink`` tokens and the ``window`` tokens ending at its
position, causally.  That is the read set of ``DSAAttention`` / CSA in the reference
(``src/linattn/variants/selection.py:738-763``: selection OR sink OR window, then the
causal intersection of ``BlockSelectionAttention.effective_mask``, ``:86-108``).

``dsa_attention`` is the config-3 pipeline: the lightning indexer's causal top-k
(``indexer_topk``, index-ordered lists) followed by the token attention over the
selected tokens, the selection shared by every head.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import lists_desc
from linattn_b200.indexer import indexer_topk

__all__ = ["token_sparse_attention", "dsa_attention"]


def token_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ids: torch.Tensor, *,
                           block: int = 1, sink: int = 0, window: int = 0, causal: bool = True, offset: int = 0,
                           scale: Optional[float] = None, counts: Optional[torch.Tensor] = None,
                           diag_fallback: bool = True, lse_out: Optional[torch.Tensor] = None,
                           reads_out: Optional[torch.Tensor] = None,
                           out: Optional[torch.Tensor] = None, v_f16: bool = True) -> torch.Tensor:
    """``q (B,H_q,T_q,D)`` over ``k, v (B,H_kv,T_k,D)``; ``ids (B,H_l,T_q,N)`` (or
    ``(B,H_l,N)`` shared by all queries) with ``H_q % H_l == 0``; negative ids are padding.
    ``diag_fallback``: a query with nothing to read reads its own position (the
    reference's empty-row rule); ``reads_out`` (B,H_q,T_q) int32 receives the number of
    tokens each query read.  ``v_f16`` (bf16 inputs, contiguous K / V): P V on an f16
    copy of V with one f16 P part (one extra pass over V)."""
    dev = L.require_cuda(q, k, v, ids, counts, lse_out, reads_out)
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape:
        raise ValueError("q must be (B,H_q,T_q,D) and k, v (B,H_kv,T_k,D) of one shape")
    b, hq, tq, d = q.shape
    hkv, tk = k.shape[1], k.shape[2]
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise ValueError("q, k and v must have one dtype (bf16 or f16)")
    if k.stride(3) != 1 or v.stride() != k.stride():
        k, v = k.contiguous(), v.contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.long()
    if ids.stride(-1) != 1:
        ids = ids.contiguous()
    lists = lists_desc(ids, ids.shape[1], counts)
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    status = L.status_word(dev)
    v_arg, v_unscale = v, None
    if q.dtype == torch.bfloat16 and v_f16 and v.is_contiguous() and k.stride() == v.stride():
        # an f16 copy of V, scaled by a power of two per (b, kv head), so that P V takes
        # one f16 P part (the scale is undone on the output)
        v_arg = torch.empty(v.shape, dtype=torch.float16, device=dev)
        v_unscale = torch.empty(b * hkv, dtype=torch.float32, device=dev)
        amax = torch.empty(b * hkv, dtype=torch.int32, device=dev)
        L.check(L.lib().linattn_prefill_v_to_f16(v.data_ptr(), b * hkv, tk * d, v_arg.data_ptr(),
                                                 v_unscale.data_ptr(), amax.data_ptr(), L.stream_of(q)))
    L.check(L.lib().linattn_token_attention(
        q.data_ptr(), L.dtype_code(q), b, hq, tq, L.strides4(q), k.data_ptr(), v_arg.data_ptr(), L.ptr(v_unscale),
        hkv, tk, d,
        (L.c_i64 * 3)(k.stride(0), k.stride(1), k.stride(2)), lists, block, sink, window, int(causal), offset, scale,
        int(diag_fallback), out.data_ptr(), L.strides4(out), L.ptr(lse_out), L.ptr(reads_out), status.data_ptr(),
        L.stream_of(q)))
    if L.strict():
        L.check_status(dev)
    return out


def dsa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_idx: torch.Tensor, k_idx: torch.Tensor,
                  head_weights: torch.Tensor, topk: int, *, k_scale: Optional[torch.Tensor] = None,
                  scale_group: int = 64, offset: int = 0, sink: int = 0, window: int = 0,
                  return_ids: bool = False):
    """Config-3 DSA prefill: causal top-``topk`` tokens per query from the lightning
    indexer (``q_idx (B,T_q,H_I,d)``, ``k_idx (B,T_k,H_I,d)``, fp8 keys with
    ``k_scale``), then attention of every head of ``q`` over its query's tokens."""
    _, ids = indexer_topk(q_idx, k_idx, head_weights, topk, causal=True, offset=offset, k_scale=k_scale,
                          scale_group=scale_group, index_dtype=torch.int32, sorted=False)
    lists = ids.unsqueeze(1)  # (B, 1, T_q, k): shared by all heads
    o = token_sparse_attention(q, k, v, lists, sink=sink, window=window, causal=True, offset=offset)
    return (o, ids) if return_ids else o
