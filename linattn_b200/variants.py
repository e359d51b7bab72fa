"""CUDA implementations of the reference's selection variants behind ``AttentionVariant``.

``CudaQuestAttention`` is the B200 counterpart of ``QuestAttention``
(``src/linattn/variants/selection.py:139-248``): same config keys
(``extras["page_size"]``, ``["gqa_union"]``, ``["dense_layers"]``, ``["layer_idx"]``,
``topk_blocks``), same state keys (``k, v, pos, page_min, page_max``,
``selection.py:169-173``), same outputs and ``stats()`` keys (``reads_per_query``,
``pages_per_query``).  The selection (page bounds, page scores, top-k, GQA union)
and the attention over the selected pages run in the sm_100a kernels; the reference's
token-level boolean mask plus full masked attention (``selection.py:86-116``) is
replaced by attention over the selected pages only, with the causal limit applied
inside the kernel.  Results agree with the reference's mask semantics: pages are
selected per query head, the group reads the union, rows after the query position
are never read, and a query always reads its own page.
"""

from __future__ import annotations

from typing import Any, Dict, Optional

import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import kv_contiguous, lists_desc, sparse_attention
from linattn_b200.core import AttentionVariant
from linattn_b200.quest_pages import page_bounds, quest_select

__all__ = ["CudaQuestAttention", "CUDA_SUPPORTED"]

CUDA_SUPPORTED = ("quest",)


class CudaQuestAttention(AttentionVariant):
    name = "cuda_quest"
    family = "cuda"
    paper = ("Tang et al., Quest (ICML 2024)", "https://arxiv.org/abs/2406.10774")

    def __init__(self, cfg=None, **kw):
        super().__init__(cfg, **kw)
        ex = self.cfg.extras
        self.dense_layers = int(ex.get("dense_layers", 2))
        self.layer_idx = int(ex.get("layer_idx", 2))
        self.page_size = int(ex.get("page_size", self.cfg.block_size))
        self.gqa_union = bool(ex.get("gqa_union", True))
        self.sink_pages = int(ex.get("sink_pages", 0))
        self._reads: Optional[torch.Tensor] = None
        self._pages: Optional[torch.Tensor] = None

    # -- state ---------------------------------------------------------------------
    def prepare_state(self, batch, device, dtype) -> Dict[str, Any]:
        state = super().prepare_state(batch, device, dtype)
        z = torch.zeros(batch, self.cfg.n_kv_heads, 0, self.cfg.head_dim, device=device, dtype=dtype)
        state["page_min"] = z
        state["page_max"] = z.clone()
        return state

    def push_kv(self, state, k, v):
        start = state["k"].shape[-2]
        state = super().push_kv(state, k, v)
        self._refresh_pages(state, start)
        return state

    def _refresh_pages(self, state, from_pos: int) -> None:
        """Recompute the bounds of the pages touched by the new keys
        (``selection.py:181-201``) with the page-bounds kernel."""
        p = self.page_size
        k = state["k"]
        t = k.shape[-2]
        first = from_pos // p
        if (t + p - 1) // p <= first:
            return
        mins, maxs = page_bounds(k[:, :, first * p:], p)
        if first == 0:
            state["page_min"], state["page_max"] = mins, maxs
        else:
            state["page_min"] = torch.cat([state["page_min"][..., :first, :], mins], dim=-2)
            state["page_max"] = torch.cat([state["page_max"][..., :first, :], maxs], dim=-2)

    # -- selection + attention -------------------------------------------------------
    def attend(self, q: torch.Tensor, state: Dict[str, Any], offset: int = 0) -> torch.Tensor:
        L.require_cuda(q)
        k, v = state["k"], state["v"]
        b, hq, tq, d = q.shape
        tk = k.shape[-2]
        p = self.page_size
        n_pages = (tk + p - 1) // p
        if k.stride(3) != 1 or k.stride(2) != d:
            k = k.contiguous()
            v = v.contiguous()
        kv = kv_contiguous(k, v, p)
        if self.layer_idx < self.dense_layers:
            ids = torch.arange(n_pages, dtype=torch.int32, device=q.device).view(1, 1, n_pages)
            ids = ids.expand(b, self.cfg.n_kv_heads, n_pages)
            out = sparse_attention(q, kv, lists_desc(ids, self.cfg.n_kv_heads), causal=True, offset=offset)
            self._reads = torch.clamp(torch.arange(tq, device=q.device) + offset + 1, max=tk).float()
            self._pages = None
            return out
        mins, maxs = state["page_min"], state["page_max"]
        group = self.group_size if self.gqa_union else 1
        meta = L.Meta(mins.data_ptr(), maxs.data_ptr(), mins.stride(0), mins.stride(2), mins.stride(1), None, 0, 0,
                      L.dtype_code(mins), mins.shape[1])
        sel = quest_select(q, meta, page_size=p, n_pages=n_pages, topk=self.cfg.topk_blocks, offset=offset,
                           sink_pages=self.sink_pages, group=group, seq_len=tk, ids_dtype=torch.int32)
        n_lists = hq // group
        lists = lists_desc(sel.union_ids, n_lists, sel.union_count)
        out = sparse_attention(q, kv, lists, causal=True, offset=offset)
        self._reads = sel.union_tokens
        self._pages = sel.union_count
        return out

    def stats(self) -> Dict[str, float]:
        out: Dict[str, float] = {}
        if self._reads is not None:
            out["reads_per_query"] = float(self._reads.float().mean())
        if self._pages is not None:
            out["pages_per_query"] = float(self._pages.float().mean())
        return out

    # -- cost model (QuestAttention / BlockSelectionAttention formulas) ---------------
    def read_budget(self, seq_len: int, batch: int = 1) -> float:
        return float(min(seq_len, self.cfg.topk_blocks * self.cfg.block_size + self.cfg.window_size))

    def selection_flops(self, seq_len: int, batch: int = 1) -> int:
        n_pages = (seq_len + self.page_size - 1) // self.page_size
        return int(2 * batch * self.cfg.n_heads * seq_len * n_pages * self.cfg.head_dim)

    def flops(self, seq_len: int, batch: int = 1) -> int:
        reads = self.read_budget(seq_len, batch)
        return int(2 * 2 * batch * self.cfg.n_heads * seq_len * reads * self.cfg.head_dim
                   + self.selection_flops(seq_len, batch))
