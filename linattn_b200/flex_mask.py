"""Block-mask views of a selection, and the check that they cover a token mask.

Mirrors ``src/linattn/kernels/flex_mask.py`` (``mask_to_block_mask``:35-47,
``to_block_mask``:50-60, ``check_block_mask``:63-72): FlexAttention's ``BlockMask``
describes which query blocks read which key blocks, and a selection expressed at that
granularity must be a superset of the variant's token mask or reads are silently
dropped.  ``lists_to_block_mask`` gives the same view of this library's block lists
(ascending ids, -1 padded, optional counts: what ``block_select``, ``moba_select``,
the Quest union lists and ``window_block_select`` produce), so a selection can be
checked against the token mask it is meant to serve.  These are validation
utilities (torch ops on whatever device the tensors live on), not part of the
attention path.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

__all__ = ["flex_available", "mask_to_block_mask", "to_block_mask", "check_block_mask", "lists_to_block_mask",
           "check_lists_cover"]


def flex_available() -> bool:
    try:
        from torch.nn.attention.flex_attention import flex_attention  # noqa: F401

        return True
    except Exception:
        return False


def mask_to_block_mask(mask: torch.Tensor, q_block: int, k_block: int) -> torch.Tensor:
    """Token mask ``(B, H, T_q, T_k)`` -> block mask ``(B, H, n_qb, n_kb)``: a block is
    kept when any query of the query block reads any key of the key block."""
    b, h, t_q, t_k = mask.shape
    n_qb, n_kb = -(-t_q // q_block), -(-t_k // k_block)
    padded = torch.zeros(b, h, n_qb * q_block, n_kb * k_block, dtype=torch.bool, device=mask.device)
    padded[..., :t_q, :t_k] = mask.bool()
    return padded.view(b, h, n_qb, q_block, n_kb, k_block).any(-3).any(-1)


def to_block_mask(mask: torch.Tensor, q_block: int = 64, k_block: int = 64):
    """A ``torch.nn.attention.flex_attention.BlockMask`` of ``mask_to_block_mask``."""
    from torch.nn.attention.flex_attention import create_block_mask

    reduced = mask_to_block_mask(mask, q_block, k_block)
    b, h, n_qb, n_kb = reduced.shape

    def mask_mod(batch, head, q_idx, kv_idx):
        return reduced[batch, head, q_idx, kv_idx]

    return create_block_mask(mask_mod, B=b, H=h, Q_LEN=n_qb, KV_LEN=n_kb, device=mask.device)


def check_block_mask(mask: torch.Tensor, reduced: torch.Tensor, q_block: int, k_block: int) -> Tuple[bool, float]:
    """``(ok, coverage)``: ``ok`` when the block mask, expanded to tokens, holds every
    token the mask reads; ``coverage`` is the fraction of blocks kept (well above the
    token mask's own density means the block granularity wastes reads)."""
    full = reduced.bool().repeat_interleave(q_block, dim=-2).repeat_interleave(k_block, dim=-1)
    full = full[..., : mask.shape[-2], : mask.shape[-1]]
    ok = bool((mask.bool() & ~full).sum() == 0)
    return ok, float(reduced.float().mean())


def lists_to_block_mask(ids: torch.Tensor, n_kb: int, counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block lists ``ids (B, H, R, N)`` (one list per row: a query block, or a query
    for per-token routing; entries < 0, past ``counts`` or >= ``n_kb`` ignored) ->
    ``(B, H, R, n_kb)`` bool."""
    b, h, r, n = ids.shape
    valid = (ids >= 0) & (ids < n_kb)
    if counts is not None:
        valid &= torch.arange(n, device=ids.device) < counts.to(ids.device)[..., None]
    out = torch.zeros(b, h, r, n_kb + 1, dtype=torch.bool, device=ids.device)
    out.scatter_(-1, torch.where(valid, ids.long(), torch.full_like(ids, n_kb, dtype=torch.long)), True)
    return out[..., :n_kb]


def check_lists_cover(mask: torch.Tensor, ids: torch.Tensor, k_block: int, counts: Optional[torch.Tensor] = None,
                      rows_per_list: int = 64) -> Tuple[bool, float]:
    """``check_block_mask`` of block lists against a token mask ``(B, H, T_q, T_k)``:
    each list serves ``rows_per_list`` consecutive queries (64 for per-q-block lists, 1
    for per-token routing) and names key blocks of ``k_block`` tokens."""
    n_kb = -(-mask.shape[-1] // k_block)
    return check_block_mask(mask, lists_to_block_mask(ids, n_kb, counts), rows_per_list, k_block)
