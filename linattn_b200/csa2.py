"""CSA2 compressed sparse attention on the sm_100a kernels (``CSA2Attention``,
``src/linattn/variants/csa2.py``).

Same parameters (``q_proj (H, E, d, F)`` drawn from ``cfg.seed`` as the reference
draws it, ``head_weights = 1/E``), config keys (``extras["compress_ratio"]``,
``["topk_groups"]``, ``["bits"]``, ``["quant_group"]``, ``["cross_layer_group"]``,
``["window"]``, ``["indexer_heads"]``, ``["indexer_dim"]``), outputs and ``stats()``
keys (``reads_per_query``, ``groups_per_query``, ``tokens_equivalent``, ``bits``).

Pipeline per ``attend``:

1. ``csa2_pool_quant`` (one kernel per k / v): mean of each group of ``compress_ratio``
   tokens, rounded to the cache dtype, stored through the FP4 / FP8 group codec and
   dequantised (``compressed_kv``, ``csa2.py:73-81``; codes bit-identical to the
   reference's);
2. the lightning-indexer projections (small torch einsums, as in the reference) and the
   indexer score + top-k kernels over the pooled groups.  A group is eligible when it
   ends before the query's raw window ``[p - w + 1, p]`` (``csa2.py:107-112``); that is
   the indexer's causal key-block rule (group g visible while ``g * m <= pos``) with the
   query positions shifted by ``1 - w - m``, so the top-k never sees an ineligible group
   and rows with fewer eligible groups than ``topk_groups`` pad with -1 (the reference
   takes top-k over -inf scores and intersects with eligibility: the same read set);
3. one softmax over the raw window plus the selected groups, the pooled rows appended
   after the raw keys (``csa2.py:122-130``): the token-sparse kernel (bf16 / f16, head
   sizes 64 / 128) with the window as its window range and the groups as listed tokens,
   otherwise the general sparse kernel over explicit per-query token lists.
"""

from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import kv_contiguous, lists_desc, sparse_attention
from linattn_b200.core import AttentionVariant
from linattn_b200.dsa import token_sparse_attention
from linattn_b200.indexer import indexer_topk

__all__ = ["csa2_pool_quant", "CudaCSA2Attention"]


def csa2_pool_quant(x: torch.Tensor, ratio: int, bits: int = 4, group: int = 32,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x (B, H, T, D)`` (bf16 / f16 / f32, any strides) -> ``(B, H, ceil(T / ratio), D)``
    contiguous in x's dtype: the group means rounded to the dtype, then for ``bits`` 4 /
    8 quantised with one absmax scale per ``group`` (= 32) channels and dequantised
    (``block_reduce``, ``src/linattn/core.py:103-120``; ``quantize`` / ``dequantize``,
    ``src/linattn/kv/quant.py:76-109``)."""
    L.require_cuda(x)
    if x.dim() != 4:
        raise ValueError("x must be (B, H, T, D)")
    if bits not in (4, 8, 16):
        raise ValueError("bits must be 4, 8 or 16")
    b, h, t, d = x.shape
    g = -(-t // ratio) if ratio >= 1 else 0
    if out is None:
        out = torch.empty(b, h, g, d, dtype=x.dtype, device=x.device)
    L.check(L.lib().linattn_csa2_pool_quant(x.data_ptr(), L.dtype_code(x), b, h, t, d, L.strides4(x), int(ratio),
                                             int(bits), int(group), out.data_ptr(), L.stream_of(x)))
    return out


class CudaCSA2Attention(AttentionVariant):
    name = "cuda_csa2"
    family = "cuda"
    paper = ("DeepSeek-AI, DeepSeek-V4.1-Flash: CSA2 + FP4 KV (2026)", "https://arxiv.org/abs/2609.19969")

    def __init__(self, cfg=None, **kw):
        super().__init__(cfg, **kw)
        ex = self.cfg.extras
        self.compress_ratio = int(ex.get("compress_ratio", self.cfg.compress_ratio))
        self.topk_groups = int(ex.get("topk_groups", self.cfg.topk_blocks))
        self.bits = int(ex.get("bits", 4))
        self.quant_group = int(ex.get("quant_group", 32))
        self.cross_layer_group = int(ex.get("cross_layer_group", 1))
        self.window = int(ex.get("window", self.cfg.window_size))
        self.n_indexer_heads = int(ex.get("indexer_heads", 4))
        self.indexer_dim = int(ex.get("indexer_dim", 16))
        if self.bits not in (4, 8, 16):
            raise ValueError("bits must be 4, 8 or 16")
        gen = torch.Generator().manual_seed(self.cfg.seed)
        self.q_proj = torch.nn.Parameter(
            torch.randn(self.cfg.n_heads, self.n_indexer_heads, self.cfg.head_dim, self.indexer_dim,
                        generator=gen) * 0.02)
        self.head_weights = torch.nn.Parameter(torch.full((self.n_indexer_heads,), 1.0 / self.n_indexer_heads))
        self._groups: Optional[torch.Tensor] = None
        self._window_reads: Optional[torch.Tensor] = None

    @property
    def storage_precision(self) -> str:
        return f"fp{self.bits} compressed + fp16 window"

    # -- storage ---------------------------------------------------------------------
    def compressed_kv(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Pooled, stored-precision keys and values in the cache dtype (``csa2.py:73-81``)."""
        return (csa2_pool_quant(k, self.compress_ratio, self.bits, self.quant_group),
                csa2_pool_quant(v, self.compress_ratio, self.bits, self.quant_group))

    def indexer_scores(self, q: torch.Tensor, kc: torch.Tensor) -> torch.Tensor:
        """``(B, H, T_q, G)`` fp32 scores of every pooled group (``csa2.py:83-92``),
        without masking; the attention path fuses them with the top-k instead."""
        from linattn_b200.indexer import indexer_scores

        q_idx, k_idx, w_t = self._projections(q, kc)
        b, h, t_q = q.shape[:3]
        s = indexer_scores(q_idx, k_idx, w_t)
        return s.view(b, h, t_q, kc.shape[-2])

    def _projections(self, q: torch.Tensor, kc: torch.Tensor):
        b, h, t_q, _ = q.shape
        e, f = self.n_indexer_heads, self.indexer_dim
        proj = self.q_proj.detach().to(q.device, q.dtype)
        q_idx = torch.einsum("bhtd,hedf->bhtef", q, proj)
        k_idx = torch.einsum("bhtd,hedf->bhtef", kc.repeat_interleave(self.group_size, dim=1), proj)
        w = torch.softmax(self.head_weights.detach().to(q.device, q.dtype), dim=-1)
        return (q_idx.reshape(b * h, t_q, e, f), k_idx.reshape(b * h, kc.shape[-2], e, f),
                w.view(1, 1, e).expand(b * h, t_q, e))

    def select_groups(self, q: torch.Tensor, kc: torch.Tensor, t_k: int, offset: int) -> torch.Tensor:
        """Selected pooled groups ``(B, H, T_q, keep)`` int32, ascending, -1 padded:
        the top ``max(1, min(topk_groups, G))`` eligible groups (``csa2.py:107-120``)."""
        b, h, t_q, _ = q.shape
        m, n_groups = self.compress_ratio, kc.shape[-2]
        win = max(1, min(self.window, t_k))
        keep = max(1, min(self.topk_groups, n_groups))
        q_idx, k_idx, w_t = self._projections(q, kc)
        _, ids = indexer_topk(q_idx, k_idx, w_t, keep, causal=True, offset=offset + 1 - win - m, key_block=m,
                              index_dtype=torch.int32, sorted=False)
        return ids.view(b, h, t_q, -1)

    # -- attention -------------------------------------------------------------------
    def attend(self, q: torch.Tensor, state: Dict[str, Any], offset: int = 0) -> torch.Tensor:
        return self.attend_kv(q, state["k"], state["v"], offset=offset)

    def attend_kv(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, offset: int = 0,
                  compressed: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
        """``attend`` over explicit ``k, v``; ``compressed = (kc, vc)`` is this k, v's
        ``compressed_kv`` when the caller already holds it (cross-layer reuse: every layer
        of a group reads the representative layer's copy)."""
        L.require_cuda(q)
        b, h, t_q, d = q.shape
        t_k = k.shape[-2]
        win = max(1, min(self.window, t_k))
        kc, vc = self.compressed_kv(k, v) if compressed is None else compressed
        gids = self.select_groups(q, kc, t_k, offset)
        gids = torch.where(gids >= 0, gids + t_k, gids)  # pooled rows follow the raw keys
        k_all = torch.cat([k, kc], dim=-2)
        v_all = torch.cat([v, vc], dim=-2)
        pos = torch.arange(t_q, device=q.device) + offset
        if q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype and d in (64, 128):
            reads = torch.empty(b, h, t_q, dtype=torch.int32, device=q.device)
            out = token_sparse_attention(q, k_all, v_all, gids, block=1, sink=0, window=win, causal=False,
                                         offset=offset, diag_fallback=False, reads_out=reads)
        else:
            wk = (pos - win + 1)[:, None] + torch.arange(win, device=q.device)
            wk = torch.where((wk >= 0) & (wk < t_k), wk, torch.full_like(wk, -1)).to(torch.int32)
            lists = torch.cat([wk.expand(b, h, t_q, win), gids], dim=-1).contiguous()
            out = sparse_attention(q, kv_contiguous(k_all.contiguous(), v_all.contiguous(), 1),
                                   lists_desc(lists, h), causal=False, offset=offset)
            reads = (lists >= 0).sum(-1)
        self._window_reads = (torch.clamp(pos, max=t_k - 1) - torch.clamp(pos - win + 1, min=0) + 1).clamp(min=0)
        self._groups = reads - self._window_reads
        return out

    def stats(self, rows: Optional[slice] = None) -> Dict[str, float]:
        """The last ``attend``'s means; ``rows`` restricts them to a range of its queries."""
        if self._groups is None:
            return {}
        sel = slice(None) if rows is None else rows
        groups = float(self._groups[..., sel].double().mean())
        window_reads = float(self._window_reads[sel].double().mean())
        return {"reads_per_query": groups + window_reads, "groups_per_query": groups,
                "tokens_equivalent": groups * self.compress_ratio + window_reads, "bits": float(self.bits)}

    # -- accounting (CSA2Attention formulas, csa2.py:148-161) --------------------------
    def _quant_bytes(self, n_values: int) -> float:
        if self.bits >= 16:
            return n_values * 2.0
        return n_values * self.bits / 8.0 + math.ceil(n_values / self.quant_group) * 2.0

    def read_budget(self, seq_len: int, batch: int = 1) -> float:
        groups = max(1, min(self.topk_groups, (seq_len + self.compress_ratio - 1) // self.compress_ratio))
        return float(groups + min(self.window, seq_len))

    def memory_bytes(self, seq_len: int, batch: int = 1) -> int:
        n_groups = (seq_len + self.compress_ratio - 1) // self.compress_ratio
        compressed = 2 * self.cfg.n_kv_heads * n_groups * self.cfg.head_dim
        raw_window = 2 * self.cfg.n_kv_heads * min(self.window, seq_len) * self.cfg.head_dim
        return int((self._quant_bytes(compressed) + raw_window * 2) * batch / self.cross_layer_group)

    def selection_flops(self, seq_len: int, batch: int = 1) -> int:
        n_groups = (seq_len + self.compress_ratio - 1) // self.compress_ratio
        return int(2 * batch * self.cfg.n_heads * seq_len * n_groups * self.indexer_dim)

    def flops(self, seq_len: int, batch: int = 1) -> int:
        reads = self.read_budget(seq_len, batch)
        return int(2 * 2 * batch * self.cfg.n_heads * seq_len * reads * self.cfg.head_dim
                   + self.selection_flops(seq_len, batch))
