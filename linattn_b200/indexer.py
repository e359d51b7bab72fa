"""Lightning-indexer scores and top-k on the B200 (DSA / CSA token selection).

``indexer_topk(q_idx, k_idx, head_weights, k, *, backend)`` keeps the signature and
semantics of ``src/linattn/kernels/triton/fused_indexer.py:197-206`` (and of its
torch reference ``indexer_topk_torch``, ``:63-73``):
``I[b,t,s] = sum_h w[b,t,h] * ReLU(q_idx[b,t,h,:] . k_idx[b,s,h,:])``, ``k = min(k, T_k)``,
values descending.  Differences, all documented: values are fp32 whatever the input
dtype (the kernel accumulates in fp32); ties go to the lowest key index (torch.topk
leaves their order unspecified); ``causal=True`` masks keys after ``offset + t`` before
the top-k and pads slots past the visible count with (-inf, -1); ``k_scale`` takes fp8
e4m3 keys with one fp32 scale per ``scale_group`` tokens.

The scores of a chunk of queries go to a scratch buffer (at most ``max_scratch_bytes``)
and each row is reduced by the radix-select top-k kernel; the full ``T_q x T_k``
matrix is never materialised.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from linattn_b200 import _lib as L

__all__ = ["indexer_scores", "indexer_topk", "row_topk", "quantize_keys_fp8"]

_MAX_SCRATCH = 1 << 29  # 512 MiB of fp32 scores per chunk


def _checked(q_idx, k_idx, head_weights, k_scale, scale_group):
    L.require_cuda(q_idx, k_idx, head_weights, k_scale)
    if q_idx.dim() != 4 or k_idx.dim() != 4 or head_weights.dim() != 3:
        raise ValueError("q_idx must be (B,T_q,H_I,D), k_idx (B,T_k,H_I,D), head_weights (B,T_q,H_I)")
    b, tq, h, d = q_idx.shape
    if k_idx.shape[0] != b or k_idx.shape[2] != h or k_idx.shape[3] != d:
        raise ValueError(f"k_idx shape {tuple(k_idx.shape)} does not match q_idx {tuple(q_idx.shape)}")
    if tuple(head_weights.shape) != (b, tq, h):
        raise ValueError(f"head_weights must be (B,T_q,H_I) = {(b, tq, h)}")
    fp8 = k_idx.dtype in (torch.float8_e4m3fn, torch.uint8)
    if fp8:
        if k_scale is None:
            raise ValueError("fp8 keys need k_scale (B, ceil(T_k / scale_group))")
        n_groups = -(-k_idx.shape[1] // scale_group)
        if k_scale.dtype != torch.float32 or k_scale.dim() != 2 or k_scale.shape[0] != b \
                or k_scale.shape[1] < n_groups or k_scale.stride(1) != 1:
            raise ValueError(f"k_scale must be fp32 (B, >= {n_groups}) with unit stride on the token axis")
    elif k_scale is not None:
        raise ValueError("k_scale is only used with fp8 keys")
    return b, tq, k_idx.shape[1], h, d, fp8


def _launch_scores(q_idx, k_idx, head_weights, k_scale, scale_group, causal, offset, t0, t1, out, row_stride,
                   key_block=1):
    b, tq, h, d = q_idx.shape
    tk = k_idx.shape[1]
    s = k_scale.stride(0) if k_scale is not None else 0
    L.check(L.lib().linattn_indexer_scores(
        q_idx.data_ptr(), L.dtype_code(q_idx), L.strides4(q_idx), k_idx.data_ptr(), L.dtype_code(k_idx),
        L.strides4(k_idx), L.ptr(k_scale), scale_group, s, head_weights.data_ptr(), L.dtype_code(head_weights),
        (L.c_i64 * 3)(*head_weights.stride()), b, tq, tk, h, d, int(causal), offset, key_block, t0, t1,
        out.data_ptr(),
        row_stride, L.status_word(q_idx.device).data_ptr(), L.stream_of(q_idx)))


def indexer_scores(q_idx: torch.Tensor, k_idx: torch.Tensor, head_weights: torch.Tensor, *,
                   k_scale: Optional[torch.Tensor] = None, scale_group: int = 64, causal: bool = False,
                   offset: int = 0, key_block: int = 1) -> torch.Tensor:
    """``(B,T_q,T_k)`` fp32 indexer scores (``fused_indexer.py:52-60``); with ``causal``,
    -inf at keys ``s`` with ``s * key_block > offset + t`` (``key_block`` > 1: keys are
    pooled groups of that many tokens)."""
    b, tq, tk, _, _, _ = _checked(q_idx, k_idx, head_weights, k_scale, scale_group)
    out = torch.empty(b, tq, tk, dtype=torch.float32, device=q_idx.device)
    if out.numel():
        _launch_scores(q_idx, k_idx, head_weights, k_scale, scale_group, causal, offset, 0, tq, out, tk, key_block)
    return out


def indexer_topk(q_idx: torch.Tensor, k_idx: torch.Tensor, head_weights: torch.Tensor, k: int, *,
                 backend: str = "auto", causal: bool = False, offset: int = 0,
                 k_scale: Optional[torch.Tensor] = None, scale_group: int = 64,
                 index_dtype: torch.dtype = torch.int64, sorted: bool = True, key_block: int = 1,
                 max_scratch_bytes: int = _MAX_SCRATCH) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-``k`` indexer scores per query: ``(values fp32 (B,T_q,k'), indices (B,T_q,k'))``
    with ``k' = min(k, T_k)`` (``fused_indexer.py:197-206``).  ``sorted=False`` returns
    the same set in ascending index order (the order the sparse attention reads it in)."""
    if backend not in ("auto", "cuda"):
        raise ValueError(f"linattn_b200 has one backend ('cuda'); got backend={backend!r}")
    if index_dtype not in (torch.int32, torch.int64):
        raise ValueError("index_dtype must be torch.int32 or torch.int64")
    b, tq, tk, _, _, _ = _checked(q_idx, k_idx, head_weights, k_scale, scale_group)
    kk = min(int(k), tk)
    if kk < 1 and tk > 0:
        raise ValueError("k must be >= 1")
    dev = q_idx.device
    values = torch.empty(b, tq, kk, dtype=torch.float32, device=dev)
    indices = torch.empty(b, tq, kk, dtype=index_dtype, device=dev)
    if values.numel() == 0:
        return values, indices
    rows = max(1, min(tq, max_scratch_bytes // max(1, b * tk * 4)))
    scratch = torch.empty(b * rows * tk, dtype=torch.float32, device=dev)
    i64 = index_dtype == torch.int64
    for t0 in range(0, tq, rows):
        t1 = min(tq, t0 + rows)
        # causal mode 2: score tiles after every query of a block are never read
        _launch_scores(q_idx, k_idx, head_weights, k_scale, scale_group, 2 if causal else 0, offset, t0, t1,
                       scratch, tk, key_block)
        v = values[:, t0]
        ix = indices[:, t0]
        L.check(L.lib().linattn_row_topk(
            scratch.data_ptr(), b * (t1 - t0), tk, tk, kk, int(causal), offset + t0, key_block, t1 - t0, 0, int(sorted),
            v.data_ptr(), ix.data_ptr() if i64 else None, None if i64 else ix.data_ptr(), kk, tq * kk,
            L.stream_of(q_idx)))
    if L.strict():
        L.check_status(dev)
    return values, indices


def row_topk(scores: torch.Tensor, k: int, *, sorted: bool = True, causal: bool = False, first_pos: int = 0,
             key_block: int = 1, period: Optional[int] = None, skip: int = 0,
             index_dtype: torch.dtype = torch.int64) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-``k`` of each row of a 2-D fp32 ``scores`` (``torch.topk(scores, k, dim=-1)`` with
    the lowest index first among equal values).  ``sorted=False`` gives the same set in
    ascending index order.  ``causal``: row ``r`` only considers its first
    ``(first_pos + r % period) // key_block + 1`` entries; ``skip``: entries before it
    are never candidates; slots past the candidate count hold (-inf, -1)."""
    L.require_cuda(scores)
    if scores.dim() != 2 or scores.dtype != torch.float32 or scores.stride(1) != 1:
        raise ValueError("scores must be a 2-D fp32 tensor with unit stride on the last axis")
    rows, n = scores.shape
    kk = min(int(k), n)
    values = torch.empty(rows, kk, dtype=torch.float32, device=scores.device)
    indices = torch.empty(rows, kk, dtype=index_dtype, device=scores.device)
    if values.numel() == 0:
        return values, indices
    i64 = index_dtype == torch.int64
    per = max(rows, 1) if period is None else period
    L.check(L.lib().linattn_row_topk(
        scores.data_ptr(), rows, n, scores.stride(0), kk, int(causal), first_pos, key_block, per, skip, int(sorted),
        values.data_ptr(), indices.data_ptr() if i64 else None, None if i64 else indices.data_ptr(), kk, per * kk,
        L.stream_of(scores)))
    return values, indices


def quantize_keys_fp8(k_idx: torch.Tensor, group: int = 64) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp8 e4m3 indexer keys with one fp32 scale per ``group`` tokens of each batch row:
    ``scale = max(absmax, 1e-8) / 448``, ``codes = (x / scale).to(float8_e4m3fn)``
    (the codec of ``src/linattn/kv/quant.py:76-109`` grouped along the token axis).
    Returns ``(codes (B,T_k,H_I,D) float8_e4m3fn, scales (B, ceil(T_k/group)) fp32)``."""
    b, tk, h, d = k_idx.shape
    n_groups = -(-tk // group)
    pad = n_groups * group - tk
    x = k_idx.float()
    if pad:
        x = torch.cat([x, x.new_zeros(b, pad, h, d)], dim=1)
    xg = x.view(b, n_groups, group * h * d)
    amax = xg.abs().amax(-1).clamp_min(1e-8)
    # a true division (torch turns division by a Python scalar on CUDA into a
    # multiplication by its reciprocal, which can differ in the last bit)
    scales = amax / torch.full_like(amax, 448.0)
    codes = (xg / scales[..., None]).to(torch.float8_e4m3fn).view(b, n_groups * group, h, d)[:, :tk]
    return codes.contiguous(), scales.contiguous()

