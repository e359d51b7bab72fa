"""Block-sparse / paged attention over selected KV blocks on the B200.

``block_sparse_attention(q, k, v, block_ids, *, block_size, backend)`` keeps the
signature and semantics of ``src/linattn/kernels/triton/block_sparse.py:131-163``
(and of its torch reference ``:40-75``): each query attends to every token of its kv
head's listed blocks, positions ``>= T_k`` are masked, there is no causal mask (the
selector's job), duplicated ids count twice, the scale is ``1/sqrt(D)`` and the
output has ``q``'s dtype.  ``block_ids`` is ``(B,H_kv,N)`` (shared by all queries) or
``(B,H_kv,T_q,N)``; negative ids are treated as padding.

``sparse_attention(...)`` is the general entry: paged pools, per-list counts, causal
limits, per-query-head lists and split-KV with the ``(o, lse)`` merge.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from linattn_b200 import _lib as L

__all__ = ["block_sparse_attention", "sparse_attention", "kv_contiguous", "lists_desc", "choose_splits"]

_TILE_ROWS = {1: 64, 2: 64, 4: 64}


def tile_rows(elem_bytes: int, head_dim: int) -> int:
    return min(64, 16384 // (head_dim * elem_bytes))


def kv_contiguous(k: torch.Tensor, v: torch.Tensor, block_size: int) -> L.KV:
    """Descriptor of the reference's contiguous ``(B, H_kv, T, D)`` cache with pages of
    ``block_size`` rows (``page p of (b, h) = K[b, h, p*P:(p+1)*P]``)."""
    if k.shape != v.shape or k.stride() != v.stride() or k.dtype != v.dtype:
        raise ValueError("k and v must have the same shape, strides and dtype")
    b, h, t, d = k.shape
    if k.stride(3) != 1 or k.stride(2) != d:
        raise ValueError("k/v rows must be contiguous (stride (.., .., D, 1))")
    return L.KV(k.data_ptr(), v.data_ptr(), k.stride(0), block_size * d, k.stride(1), None, 0, 0, None, None, 0, 0,
                None, t, L.dtype_code(k), block_size, d, h)


def lists_desc(ids: torch.Tensor, n_heads: int, counts: Optional[torch.Tensor] = None) -> L.Lists:
    """Descriptor of ``ids`` shaped (B, n_heads, N) (shared over queries) or
    (B, n_heads, T_q, N)."""
    if ids.stride(-1) != 1:
        raise ValueError("block ids need unit stride on the last axis")
    if ids.dim() == 3:
        sb, sh, _ = ids.stride()
        st = 0
    elif ids.dim() == 4:
        sb, sh, st, _ = ids.stride()
    else:
        raise ValueError("block_ids must be (B,H_kv,N) or (B,H_kv,T_q,N)")
    cs = (0, 0, 0)
    if counts is not None:
        cs = counts.stride() if counts.dim() == 3 else (*counts.stride(), 0)
    return L.Lists(ids.data_ptr(), L.dtype_code(ids), n_heads, sb, sh, st, ids.shape[-1], L.ptr(counts), *cs)


def choose_splits(units: int, tiles_per_unit: int, device: torch.device) -> int:
    """Split-KV factor: enough CTAs for ~2 waves of 2 CTAs per SM, each split keeping
    at least 2 tiles of work."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    target = 4 * sms
    if units >= target or tiles_per_unit <= 2:
        return 1
    s = math.ceil(target / max(units, 1))
    return int(max(1, min(s, tiles_per_unit // 2, 64)))


def sparse_attention(q: torch.Tensor, kv: L.KV, lists: L.Lists, *, causal: bool = False, offset: int = 0,
                     scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     lse_out: Optional[torch.Tensor] = None, n_splits: Optional[int] = None,
                     workspace: Optional[torch.Tensor] = None, tiles_per_unit: Optional[int] = None,
                     _keepalive=()) -> torch.Tensor:
    """Attention of ``q (B,H_q,T_q,D)`` over the listed pages of ``kv``."""
    dev = L.require_cuda(q)
    b, hq, tq, d = q.shape
    if d != kv.head_dim:
        raise ValueError(f"head_dim mismatch: q has {d}, kv has {kv.head_dim}")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    g_total = hq // lists.n_heads
    g_t = 1
    while g_t < g_total and g_t < 8:
        g_t <<= 1
    n_hc = (g_total + g_t - 1) // g_t
    units = b * lists.n_heads * tq * n_hc
    if n_splits is None:
        if tiles_per_unit is None:
            eb = {L.F32: 4, L.F16: 2, L.BF16: 2, L.FP8E4M3: 1}[kv.dtype]
            tr = tile_rows(eb, d)
            tiles_per_unit = max(1, (lists.max_len * kv.page_size + tr - 1) // tr)
        n_splits = choose_splits(units, tiles_per_unit, dev)
    need = L.lib().linattn_sparse_attention_workspace(b, hq, tq, d, n_splits)
    if n_splits > 1 and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty((need + 3) // 4, dtype=torch.float32, device=dev)
    status = L.status_word(dev)
    L.check(L.lib().linattn_sparse_attention(
        q.data_ptr(), L.dtype_code(q), b, hq, tq, L.strides4(q), kv, lists, int(causal), offset, scale,
        out.data_ptr(), L.strides4(out), L.ptr(lse_out), n_splits, L.ptr(workspace) if n_splits > 1 else None,
        need, status.data_ptr(), L.stream_of(q)))
    if L.strict():
        L.check_status(dev)
    return out


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_ids: torch.Tensor, *,
                           block_size: Optional[int] = None, backend: str = "auto") -> torch.Tensor:
    """Exact attention over the selected key blocks (``block_sparse.py:131-163``).

    ``q``: ``(B,H,T_q,D)``; ``k``/``v``: ``(B,H_kv,T_k,D)``; ``block_ids``:
    ``(B,H_kv,N)`` or ``(B,H_kv,T_q,N)`` (int32 or int64).
    """
    if block_size is None:
        raise ValueError("block_size is required")
    if backend not in ("auto", "cuda"):
        raise ValueError(f"linattn_b200 has one backend ('cuda'); got backend={backend!r}")
    L.require_cuda(q, k, v, block_ids)
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError("q must be (B,H,T_q,D) and k/v (B,H_kv,T_k,D)")
    if q.shape[1] % k.shape[1]:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    if k.stride(3) != 1 or k.stride(2) != k.shape[3]:
        k = k.contiguous()
    if v.stride() != k.stride():
        v = v.contiguous()
        k = k.contiguous()
    if block_ids.dtype not in (torch.int32, torch.int64):
        block_ids = block_ids.long()
    if block_ids.stride(-1) != 1:
        block_ids = block_ids.contiguous()
    kv = kv_contiguous(k, v, block_size)
    lists = lists_desc(block_ids, k.shape[1])
    return sparse_attention(q, kv, lists, causal=False)
