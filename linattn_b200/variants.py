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
from linattn_b200.dsa import token_sparse_attention
from linattn_b200.indexer import indexer_topk
from linattn_b200.quest_pages import page_bounds, quest_select

__all__ = ["CudaQuestAttention", "CudaDSAAttention", "CUDA_SUPPORTED"]

CUDA_SUPPORTED = ("quest", "dsa", "csa2", "nsa")


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


def _block_mean(x: torch.Tensor, block: int) -> torch.Tensor:
    """Mean over non-overlapping blocks of the token axis (-2), the tail padded by
    repeating the last row (``block_reduce``, ``src/linattn/core.py:103-120``)."""
    if block == 1:
        return x
    t = x.shape[-2]
    pad = (-t) % block
    if pad:
        x = torch.cat([x, x[..., -1:, :].expand(*x.shape[:-2], pad, x.shape[-1])], dim=-2)
    return x.reshape(*x.shape[:-2], x.shape[-2] // block, block, x.shape[-1]).mean(dim=-2)


def _union_token_lists(ids: torch.Tensor, block: int, sink: int, window: int, t_k: int, offset: int) -> torch.Tensor:
    """The token-sparse kernel's read set as explicit per-query token lists, for the
    general sparse kernel (dtypes / head sizes the token kernel does not take): list
    tokens outside the sink and window ranges, then the sink tokens, then the window
    tokens, all causal; a query with nothing left reads min(offset + t, T_k - 1).
    ``ids (B,H,T_q,n)`` int32 (-1 padded) -> ``(B,H,T_q,n*block + sink + window)`` int32."""
    b, h, t_q, n = ids.shape
    dev = ids.device
    pos = torch.arange(t_q, device=dev) + offset
    limit = torch.clamp(pos + 1, max=t_k)
    n_sink = torch.clamp(limit, max=sink)
    w_end = limit if window > 0 else torch.zeros_like(limit)
    w_lo = torch.maximum(n_sink, pos - window + 1)
    idl = ids.long()
    tok = (idl.unsqueeze(-1) * block + torch.arange(block, device=dev)).reshape(b, h, t_q, n * block)
    ok = (idl >= 0).unsqueeze(-1).expand(b, h, t_q, n, block).reshape(b, h, t_q, n * block)
    ok = ok & (tok < limit[:, None]) & (tok >= n_sink[:, None]) & ~((tok >= w_lo[:, None]) & (tok < w_end[:, None]))
    tok = torch.where(ok, tok, torch.full_like(tok, -1))
    sk = torch.arange(sink, device=dev).expand(t_q, sink)
    sk = torch.where(sk < n_sink[:, None], sk, torch.full_like(sk, -1))
    wk = w_lo[:, None] + torch.arange(window, device=dev)
    wk = torch.where(wk < w_end[:, None], wk, torch.full_like(wk, -1))
    lists = torch.cat([tok, sk.expand(b, h, t_q, sink), wk.expand(b, h, t_q, window)], dim=-1)
    empty = (lists < 0).all(-1)
    diag = torch.clamp(pos, max=t_k - 1).view(1, 1, t_q).expand(b, h, t_q)
    lists[..., 0] = torch.where(empty, diag, lists[..., 0])
    return lists.to(torch.int32).contiguous()


class CudaDSAAttention(AttentionVariant):
    """DeepSeek Sparse Attention / CSA (``DSAAttention``, ``selection.py:659-763``).

    Same parameters (``q_proj (H, E, d, F)`` drawn from ``cfg.seed`` exactly as the
    reference does, ``head_weights = 1/E``), config keys (``extras["indexer_heads"]``,
    ``["indexer_dim"]``, ``["compress_ratio"]``, ``topk_tokens``, ``sink_size``,
    ``window_size``) and read set: top-k tokens per head from the lightning indexer
    (or, with ``compress_ratio`` m > 1, the top ``topk_tokens // m`` causal groups of m
    tokens scored against mean-pooled keys) OR sink OR window, intersected with
    causality, the empty-row fallback reading the query's own position.  The indexer
    projections are small torch einsums as in the reference; the scores + top-k run in
    the indexer kernels (fp32 scores, lowest-index ties) and the attention in the
    token-sparse kernel over the selected tokens only.
    """

    name = "cuda_dsa"
    family = "cuda"
    paper = ("DeepSeek-AI, DeepSeek-V3.2 / DSA + lightning indexer (2025)",
             "https://huggingface.co/deepseek-ai/DeepSeek-V3.2")

    def __init__(self, cfg=None, **kw):
        super().__init__(cfg, **kw)
        ex = self.cfg.extras
        self.n_indexer_heads = int(ex.get("indexer_heads", 8))
        self.indexer_dim = int(ex.get("indexer_dim", 16))
        self.compress_ratio = int(ex.get("compress_ratio", self.cfg.compress_ratio))
        gen = torch.Generator().manual_seed(self.cfg.seed)
        self.q_proj = torch.nn.Parameter(
            torch.randn(self.cfg.n_heads, self.n_indexer_heads, self.cfg.head_dim, self.indexer_dim,
                        generator=gen) * 0.02)
        self.head_weights = torch.nn.Parameter(torch.full((self.n_indexer_heads,), 1.0 / self.n_indexer_heads))
        self._reads: Optional[torch.Tensor] = None

    def select_lists(self, q: torch.Tensor, k: torch.Tensor, offset: int):
        """Per-head selections ``(B, H, T_q, n_keep)`` int32 in ascending order (-1
        padded), and the tokens per entry (1, or the compression ratio)."""
        b, h, t_q, _ = q.shape
        m = max(1, self.compress_ratio)
        kk = _block_mean(k, m)
        t_g = kk.shape[-2]
        proj = self.q_proj.detach().to(q.device, q.dtype)
        q_idx = torch.einsum("bhtd,hedf->bhtef", q, proj)
        k_rep = kk.repeat_interleave(self.group_size, dim=1)
        k_idx = torch.einsum("bhtd,hedf->bhtef", k_rep, proj)
        w = torch.softmax(self.head_weights.detach().to(q.device, q.dtype), dim=-1)
        e, f = self.n_indexer_heads, self.indexer_dim
        w_t = w.view(1, 1, e).expand(b * h, t_q, e)
        if m > 1:
            # groups whose first token is after the query are never selected
            n_keep = max(1, self.cfg.topk_tokens // m)
            _, ids = indexer_topk(q_idx.reshape(b * h, t_q, e, f), k_idx.reshape(b * h, t_g, e, f), w_t, n_keep,
                                  causal=True, offset=offset, key_block=m, index_dtype=torch.int32, sorted=False)
        else:
            # the reference takes the top-k over every key, causality applies afterwards
            n_keep = min(self.cfg.topk_tokens, t_g)
            _, ids = indexer_topk(q_idx.reshape(b * h, t_q, e, f), k_idx.reshape(b * h, t_g, e, f), w_t, n_keep,
                                  index_dtype=torch.int32, sorted=False)
        return ids.view(b, h, t_q, -1), m

    def attend(self, q: torch.Tensor, state: Dict[str, Any], offset: int = 0) -> torch.Tensor:
        L.require_cuda(q)
        k, v = state["k"], state["v"]
        ids, m = self.select_lists(q, k, offset)
        sink, window = self.cfg.sink_size, self.cfg.window_size
        if q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype and q.shape[-1] in (64, 128):
            reads = torch.empty(q.shape[0], q.shape[1], q.shape[2], dtype=torch.int32, device=q.device)
            out = token_sparse_attention(q, k, v, ids, block=m, sink=sink, window=window, causal=True,
                                         offset=offset, diag_fallback=True, reads_out=reads)
        else:
            # other dtypes / head sizes: the same read set as explicit token lists for
            # the general sparse kernel (pages of one token)
            lists = _union_token_lists(ids, m, sink, window, k.shape[-2], offset)
            if k.stride(3) != 1 or k.stride(2) != k.shape[-1]:
                k, v = k.contiguous(), v.contiguous()
            out = sparse_attention(q, kv_contiguous(k, v, 1), lists_desc(lists, q.shape[1]), causal=True,
                                   offset=offset)
            reads = (lists >= 0).sum(-1)
        self._reads = reads
        return out

    def stats(self) -> Dict[str, float]:
        return {} if self._reads is None else {"reads_per_query": float(self._reads.float().mean())}

    # -- cost model (DSAAttention / BlockSelectionAttention formulas) ------------------
    def read_budget(self, seq_len: int, batch: int = 1) -> float:
        # BlockSelectionAttention.read_budget (selection.py:123-124), which DSA inherits
        return float(min(seq_len, self.cfg.topk_blocks * self.cfg.block_size + self.cfg.window_size))

    def selection_flops(self, seq_len: int, batch: int = 1) -> int:
        m = max(1, self.compress_ratio)
        return int(2 * batch * self.cfg.n_heads * seq_len * (seq_len // m) * self.indexer_dim)

    def flops(self, seq_len: int, batch: int = 1) -> int:
        reads = self.read_budget(seq_len, batch)
        return int(2 * 2 * batch * self.cfg.n_heads * seq_len * reads * self.cfg.head_dim
                   + self.selection_flops(seq_len, batch))
