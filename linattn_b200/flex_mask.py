"""Block-granular views of a selection and the check that a block selection covers
the token reads it stands for.

The reference's FlexAttention bridge (``src/linattn/kernels/flex_mask.py:35-72``)
exposes ``mask_to_block_mask``, ``to_block_mask`` and ``check_block_mask`` with
these names, arguments and results; they are kept for callers.  The work here is
done on coordinates instead of dense grids: a token mask is read as the list of
its ``(b, h, q, k)`` reads, each read is mapped to its ``(row, key block)`` cell,
and coverage is a membership test of those cells against the block selection,
so a check costs O(reads + selected blocks) memory, not O(T_q * T_k).  The
selection may be a dense block grid or, natively, this library's block lists
(ascending ids, -1 padded, optional counts: what ``block_select``,
``moba_select``, the Quest union lists and ``window_block_select`` produce).
Validation utilities (torch ops on the tensors' device), not the attention path.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

__all__ = ["flex_available", "mask_to_block_mask", "to_block_mask", "check_block_mask", "lists_to_block_mask",
           "check_lists_cover", "lists_to_flex_block_mask"]


def flex_available() -> bool:
    try:
        from torch.nn.attention.flex_attention import BlockMask  # noqa: F401
    except Exception:
        return False
    return True


def _read_cells(mask: torch.Tensor, q_block: int, k_block: int) -> torch.Tensor:
    """Flat cell ids ``((b * H + h) * n_qb + q // q_block) * n_kb + k // k_block`` of
    every read of a token mask ``(B, H, T_q, T_k)``, one entry per read."""
    b, h, t_q, t_k = mask.shape
    n_qb, n_kb = -(-t_q // q_block), -(-t_k // k_block)
    bi, hi, qi, ki = mask.bool().nonzero(as_tuple=True)
    return ((bi * h + hi) * n_qb + qi // q_block) * n_kb + ki // k_block


def mask_to_block_mask(mask: torch.Tensor, q_block: int, k_block: int) -> torch.Tensor:
    """Token mask ``(B, H, T_q, T_k)`` -> block mask ``(B, H, n_qb, n_kb)``: a cell is
    set when some read of the mask falls in it."""
    b, h, t_q, t_k = mask.shape
    n_qb, n_kb = -(-t_q // q_block), -(-t_k // k_block)
    grid = torch.zeros(b * h * n_qb * n_kb, dtype=torch.bool, device=mask.device)
    grid[_read_cells(mask, q_block, k_block)] = True
    return grid.view(b, h, n_qb, n_kb)


def check_block_mask(mask: torch.Tensor, reduced: torch.Tensor, q_block: int, k_block: int) -> Tuple[bool, float]:
    """``(ok, coverage)`` for a block grid ``reduced (B, H, n_qb, n_kb)``: ``ok`` when
    every read of ``mask`` lands in a set cell; ``coverage`` is the fraction of cells
    set (far above the token mask's own density means the block granularity reads
    much more than the selection needs)."""
    flat = reduced.bool().reshape(-1)
    ok = bool(flat[_read_cells(mask, q_block, k_block)].all())
    return ok, float(flat.float().mean())


def to_block_mask(mask: torch.Tensor, q_block: int = 64, k_block: int = 64):
    """A FlexAttention ``BlockMask`` holding the cells of ``mask_to_block_mask``,
    built from per-row key-block lists (``BlockMask.from_kv_blocks``)."""
    reduced = mask_to_block_mask(mask, q_block, k_block)
    n_kb = reduced.shape[-1]
    counts = reduced.sum(-1, dtype=torch.int32)
    # set cells first, in ascending key-block order (a stable sort of the negated grid)
    order = torch.sort((~reduced).to(torch.int8), dim=-1, stable=True).indices.to(torch.int32)
    return lists_to_flex_block_mask(order, counts, q_block, k_block,
                                    seq_lengths=(mask.shape[-2], mask.shape[-1]) if n_kb else None)


def _valid_entries(ids: torch.Tensor, n_kb: int, counts: Optional[torch.Tensor]) -> torch.Tensor:
    valid = (ids >= 0) & (ids < n_kb)
    if counts is not None:
        valid &= torch.arange(ids.shape[-1], device=ids.device) < counts.to(ids.device)[..., None]
    return valid


def lists_to_block_mask(ids: torch.Tensor, n_kb: int, counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block lists ``ids (B, H, R, N)`` (one list per row: a query block, or a query
    for per-token routing; entries < 0, past ``counts`` or >= ``n_kb`` ignored) ->
    ``(B, H, R, n_kb)`` bool."""
    b, h, r, n = ids.shape
    valid = _valid_entries(ids, n_kb, counts)
    rows = torch.arange(b * h * r, device=ids.device).view(b, h, r, 1).expand(b, h, r, n)
    grid = torch.zeros(b * h * r * n_kb, dtype=torch.bool, device=ids.device)
    grid[(rows * n_kb + ids.long())[valid]] = True
    return grid.view(b, h, r, n_kb)


def check_lists_cover(mask: torch.Tensor, ids: torch.Tensor, k_block: int, counts: Optional[torch.Tensor] = None,
                      rows_per_list: int = 64) -> Tuple[bool, float]:
    """``(ok, coverage)`` of block lists against a token mask ``(B, H, T_q, T_k)``
    without building either as a grid: each list serves ``rows_per_list``
    consecutive queries (64 for per-q-block lists, 1 for per-token routing).  The
    listed cells are sorted once; every read's cell is then looked up in them."""
    b, h, r, n = ids.shape
    n_kb = -(-mask.shape[-1] // k_block)
    valid = _valid_entries(ids, n_kb, counts)
    rows = torch.arange(b * h * r, device=ids.device).view(b, h, r, 1).expand(b, h, r, n)
    listed = torch.unique((rows * n_kb + ids.long())[valid])  # sorted, distinct
    need = _read_cells(mask, rows_per_list, k_block)
    if need.numel() == 0:
        ok = True
    elif listed.numel() == 0:
        ok = False
    else:
        at = torch.searchsorted(listed, need).clamp(max=listed.numel() - 1)
        ok = bool((listed[at] == need).all())
    return ok, float(listed.numel()) / float(max(1, b * h * r * n_kb))


def lists_to_flex_block_mask(ids: torch.Tensor, counts: torch.Tensor, q_block: int = 64, k_block: int = 64,
                             seq_lengths: Optional[Tuple[int, int]] = None):
    """This library's block lists as a FlexAttention ``BlockMask``: row r of the lists
    is query block r, ``counts`` the number of valid leading entries."""
    from torch.nn.attention.flex_attention import BlockMask

    if q_block != k_block:
        kw = {"BLOCK_SIZE": (q_block, k_block)}
    else:
        kw = {"BLOCK_SIZE": q_block}
    return BlockMask.from_kv_blocks(counts.to(torch.int32), ids.clamp_min(0).to(torch.int32), seq_lengths=seq_lengths,
                                    **kw)
