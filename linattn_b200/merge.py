"""Split-KV ``(o, lse)`` merge on the B200.

``o = sum_s exp(lse_s - L) o_s / sum_s exp(lse_s - L)``, ``L = max_s lse_s``; the
merged lse is ``L + log(sum_s exp(lse_s - L))``.  The reference never splits the KV
axis, so this has no reference counterpart; it is the log-sum-exp identity, checked
against attention over the union of the parts.  It merges the in-GPU KV splits and,
after an NCCL all-gather, the per-GPU partials of the sequence-sharded decode.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from linattn_b200 import _lib as L

__all__ = ["lse_combine"]


def lse_combine(o_parts: torch.Tensor, lse_parts: torch.Tensor, *, out_dtype: Optional[torch.dtype] = None,
                out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """``o_parts (S, ..., D)`` fp32 and ``lse_parts (S, ...)`` fp32 (natural log, -inf =
    empty part) -> ``(o (..., D), lse (...))``."""
    dev = L.require_cuda(o_parts, lse_parts)
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise ValueError("o_parts and lse_parts must be float32")
    if o_parts.shape[:-1] != lse_parts.shape:
        raise ValueError("lse_parts must match o_parts without the channel axis")
    o_parts = o_parts.contiguous()
    lse_parts = lse_parts.contiguous()
    s, d = o_parts.shape[0], o_parts.shape[-1]
    rows = lse_parts[0].numel() if s else 0
    out_dtype = out_dtype or torch.float32
    if out is None:
        out = torch.empty(o_parts.shape[1:], dtype=out_dtype, device=dev)
    elif not out.is_contiguous() or out.shape != o_parts.shape[1:]:
        raise ValueError("out must be contiguous with shape o_parts.shape[1:]")
    lse = torch.empty(lse_parts.shape[1:], dtype=torch.float32, device=dev)
    L.check(L.lib().linattn_lse_combine(o_parts.data_ptr(), lse_parts.data_ptr(), s, rows, d, out.data_ptr(),
                                        L.dtype_code(out), lse.data_ptr(), L.stream_of(o_parts)))
    return out, lse
