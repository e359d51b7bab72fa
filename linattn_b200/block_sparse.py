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

__all__ = ["block_sparse_attention", "sparse_attention", "kv_contiguous", "lists_desc", "plan_splits",
           "uses_tensor_cores"]

def tile_rows(elem_bytes: int, head_dim: int) -> int:
    """Rows per tile of the CUDA-core kernel (fp32 / fp8 / mixed dtypes / other D)."""
    return min(64, 16384 // (head_dim * elem_bytes))


def uses_tensor_cores(kv_dtype: int, q_dtype: int, head_dim: int, page_size: Optional[int] = None) -> bool:
    """The C ABI's dispatch rule: 16-bit KV with q of the same dtype and D in {64, 128},
    or fp8 KV with a bf16 / f16 q, D = 128 and pages of >= 32 rows, run the tensor-core
    kernel (persistent grid, 4 KiB K / V tiles per warp)."""
    if kv_dtype == L.FP8E4M3:
        return q_dtype in (L.F16, L.BF16) and head_dim == 128 and (page_size is None or page_size >= 32)
    return kv_dtype in (L.F16, L.BF16) and q_dtype == kv_dtype and head_dim in (64, 128)


def mma_tile_rows(kv_dtype: int, head_dim: int) -> int:
    """Rows per warp tile of the tensor-core kernel (4 KiB of K or V)."""
    return 4096 // (head_dim * (1 if kv_dtype == L.FP8E4M3 else 2))


def plan_splits(b: int, hq: int, tq: int, d: int, kv_dtype: int, q_dtype: int, list_heads: int, max_len: int,
                page_size: int, device: torch.device) -> int:
    """Split-KV factor for a call.

    Tensor-core path (a persistent grid of 148 SMs x 8 warps, one item at a time per
    warp; items = units x S).  When one wave fits (units x S within 90% of the 1184
    warps, with at most 128 list entries per item), S is the largest such count: a
    single wave finishes with its last item, and a wave that fills the last ~10% of the
    warps ends late (configuration 2, 128 units: 8 splits = 1024 items 98 us, 9 = 1152
    items 102-106 us, 10 = a second wave 137 us).  Otherwise the items run in waves and
    S minimises ceil(units x S / 1184) x (tiles / S + 3), the waves times an item's time
    in tiles (an item start costs about 3 tiles), each item keeping at least 4 tiles:
    configuration 5 (512 units) takes 9 splits (3.9 waves, 753 us; 8 splits 806 us,
    4 splits leave the last of 1.7 waves mostly idle).  CUDA-core path: about 4 CTAs
    per SM, each split keeping at least 2 tiles."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    g_total = hq // list_heads
    tc = uses_tensor_cores(kv_dtype, q_dtype, d, page_size)
    if tc:
        tr = mma_tile_rows(kv_dtype, d)
        units = b * list_heads * tq * ((g_total + 7) // 8)
        tiles = max(1, (max_len * page_size + tr - 1) // tr) if page_size <= tr else max_len * -(-page_size // tr)
        floor = max(1, -(-max_len // 128))  # <= 128 entries per split
        cap = max(floor, min(64, tiles // 4))
        warps = 8 * sms
        one_wave = int(0.9 * warps) // max(units, 1)
        if one_wave >= floor:
            return int(max(floor, min(one_wave, cap)))
        best, best_cost = floor, None
        for s in range(floor, cap + 1):
            cost = math.ceil(units * s / warps) * (tiles / s + 3.0)
            if best_cost is None or cost < best_cost - 1e-12:
                best, best_cost = s, cost
        return int(best)
    eb = {L.F32: 4, L.F16: 2, L.BF16: 2, L.FP8E4M3: 1}[kv_dtype]
    tr = tile_rows(eb, d)
    g_t = 1
    while g_t < g_total and g_t < 8:
        g_t <<= 1
    units = b * list_heads * tq * ((g_total + g_t - 1) // g_t)
    tiles = max(1, (max_len * page_size + tr - 1) // tr)
    target, min_tiles = 4 * sms, 2
    if units >= target or tiles < 2 * min_tiles:
        return 1
    return int(max(1, min(math.ceil(target / max(units, 1)), tiles // min_tiles, 64)))


def kv_contiguous(k: torch.Tensor, v: torch.Tensor, block_size: int) -> L.KV:
    """Descriptor of the reference's contiguous ``(B, H_kv, T, D)`` cache with pages of
    ``block_size`` rows (``page p of (b, h) = K[b, h, p*P:(p+1)*P]``)."""
    if k.shape != v.shape or k.stride() != v.stride() or k.dtype != v.dtype:
        raise ValueError("k and v must have the same shape, strides and dtype")
    b, h, t, d = k.shape
    if k.stride(3) != 1 or k.stride(2) != d:
        raise ValueError("k/v rows must be contiguous (stride (.., .., D, 1))")
    rows = min(L.rows_addressable(k, d), L.rows_addressable(v, d))
    return L.KV(k.data_ptr(), v.data_ptr(), k.stride(0), block_size * d, k.stride(1), None, 0, 0, None, None, 0, 0,
                None, t, L.dtype_code(k), block_size, d, h, rows)


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


def sparse_attention(q: torch.Tensor, kv: L.KV, lists: L.Lists, *, causal: bool = False, offset: int = 0,
                     scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     lse_out: Optional[torch.Tensor] = None, n_splits: Optional[int] = None,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of ``q (B,H_q,T_q,D)`` over the listed pages of ``kv``; ``out`` (f32,
    f16 or bf16, default q's dtype) receives the result in its own dtype."""
    dev = L.require_cuda(q)
    b, hq, tq, d = q.shape
    if d != kv.head_dim:
        raise ValueError(f"head_dim mismatch: q has {d}, kv has {kv.head_dim}")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    elif out.shape != q.shape:
        raise ValueError(f"out must have q's shape {tuple(q.shape)}, got {tuple(out.shape)}")
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    if n_splits is None:
        n_splits = plan_splits(b, hq, tq, d, kv.dtype, L.dtype_code(q), lists.n_heads, lists.max_len, kv.page_size,
                               dev)
    need = L.lib().linattn_sparse_attention_workspace(b, hq, tq, d, n_splits)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty((need + 3) // 4, dtype=torch.float32, device=dev)
    status = L.status_word(dev)
    L.check(L.lib().linattn_sparse_attention_out(
        q.data_ptr(), L.dtype_code(q), b, hq, tq, L.strides4(q), kv, lists, int(causal), offset, scale,
        out.data_ptr(), L.dtype_code(out), L.strides4(out), L.ptr(lse_out), n_splits, workspace.data_ptr(), need,
        status.data_ptr(), L.stream_of(q)))
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
