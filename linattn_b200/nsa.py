"""NSA three-branch sparse attention on the sm_100a kernels (``NSAAttention``,
``src/linattn/variants/native_sparse.py``).

Same parameters (``gates (H, 3) = 1/3 + 0.01 * randn`` drawn from ``cfg.seed``), config
keys (``extras["compress_ratio"]``, ``["selected_blocks"]``, ``["gate_mode"]``,
``block_size``, ``window_size``), ``stats()`` keys (``reads_per_query``,
``selected_blocks_per_query``), cost formulas and ``fit_gates``.  The three branches:

* compression (``native_sparse.py:67-76``): keys / values pooled by ``csa2_pool_quant``
  at 16 bits (the mean in the cache dtype, as ``block_reduce``); the groups a query
  reads are a prefix (those starting at or before ``p + c - 1``): the tcgen05 prefill
  kernel with its pooled causal rule (``causal = c``) at head size 128 in bf16 / f16,
  otherwise the shared ids ``0 .. G-1`` with a per-query count;
* selection (``:78-98``): block means of k (cache dtype), then one kernel for the fp32
  scores of every query against them, the top-k over the blocks starting at or before
  the query and the merge with the own block (``block_score_topk``); the selected
  blocks are read whole (no causal cut, as the reference's mask): the tcgen05 prefill
  kernel for 64-token blocks at head size 128 in bf16 / f16, the general sparse kernel
  otherwise;
* window (``:100-105``): the tcgen05 prefill with a token-exact window bound (head size
  128 in bf16 / f16: each 64-query block lists the key blocks its windows touch), the
  token-sparse kernel's window range (head size 64), or explicit window lists for the
  general kernel.

Each branch writes fp32; the gates combine them and round once to the output dtype.
A query with fewer allowed blocks than ``selected_blocks`` reads its allowed blocks
only; the reference's ``topk_blocks`` fills such rows with blocks starting after the
query, chosen by torch's top-k among -inf scores in no defined order.
"""

from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import kv_contiguous, lists_desc, sparse_attention
from linattn_b200.blocks import block_score_topk, block_sparse_prefill
from linattn_b200.core import AttentionVariant
from linattn_b200.csa2 import csa2_pool_quant
from linattn_b200.dsa import token_sparse_attention

__all__ = ["CudaNSAAttention", "nsa_select"]


def _token_kernel_ok(q: torch.Tensor, k: torch.Tensor) -> bool:
    return q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype and q.shape[-1] in (64, 128)


def nsa_select(q: torch.Tensor, k: torch.Tensor, block: int, selected: int, *,
               offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per (b, q-head, query) block lists of NSA's selection branch
    (``native_sparse.py:78-92``): ``(ids (B, Hq, Tq, kk + 1) int32 ascending -1 padded,
    counts (B, Hq, Tq) int32)``."""
    d = q.shape[-1]
    kp = csa2_pool_quant(k, block, 16)  # block_reduce in the cache dtype
    kk = max(1, min(selected, kp.shape[2]))
    # block j is allowed for the query at p iff j * block <= p; scores in fp32 (16-bit
    # products are exact in fp32), ranked and merged with the own block in one kernel
    return block_score_topk(q, kp, kk, scale=1.0 / math.sqrt(d), first_pos=offset, key_block=block,
                            merge_pos=offset, own_div=block, force_own=True, n_max=kk + 1)


class CudaNSAAttention(AttentionVariant):
    name = "cuda_nsa"
    family = "cuda"
    paper = ("Yuan et al., Native Sparse Attention (ACL 2025)", "https://arxiv.org/abs/2502.11089")

    def __init__(self, cfg=None, **kw):
        super().__init__(cfg, **kw)
        ex = self.cfg.extras
        self.compress = int(ex.get("compress_ratio", self.cfg.compress_ratio))
        self.selected_blocks = int(ex.get("selected_blocks", self.cfg.topk_blocks))
        self.gate_mode = ex.get("gate_mode", "uniform")
        gen = torch.Generator().manual_seed(self.cfg.seed)
        init = torch.full((self.cfg.n_heads, 3), 1.0 / 3.0)
        self.gates = torch.nn.Parameter(init + 0.01 * torch.randn(self.cfg.n_heads, 3, generator=gen))
        self._sel_counts: Optional[torch.Tensor] = None

    # -- branches --------------------------------------------------------------------
    def compressed_kv(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        return csa2_pool_quant(k, self.compress, 16), csa2_pool_quant(v, self.compress, 16)

    def branch_compression(self, q, k, v, offset: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        L.require_cuda(q)
        b, hq, tq, d = q.shape
        c = self.compress
        kc, vc = self.compressed_kv(k, v)
        hkv, n_groups = kc.shape[1], kc.shape[2]
        pos = torch.arange(tq, device=q.device) + offset
        # groups starting at or before p + c - 1: the first (p + c - 1) // c + 1
        counts = torch.clamp((pos + c - 1).div(c, rounding_mode="floor") + 1, min=1, max=n_groups)
        counts = counts.to(torch.int32).view(1, 1, tq).expand(b, hkv, tq)
        ids = torch.arange(n_groups, dtype=torch.int32, device=q.device).view(1, 1, n_groups).expand(b, hkv, n_groups)
        n_blk = -(-n_groups // 64)
        if d == 128 and q.dtype in (torch.bfloat16, torch.float16) and kc.dtype == q.dtype and n_blk <= 64:
            # tensor cores: every 128-query tile reads the pooled blocks once; the prefill
            # kernel's causal rule with c = compress_ratio is exactly this prefix
            blocks = torch.arange(n_blk, dtype=torch.int32, device=q.device).view(1, 1, 1, n_blk)
            res = block_sparse_prefill(q, kc, vc, blocks.expand(b, hq, 1, n_blk), rows_per_list=max(tq, 1),
                                       causal=c, offset=offset)
            return res if out is None else out.copy_(res)
        if _token_kernel_ok(q, kc):
            res = token_sparse_attention(q, kc, vc, ids, counts=counts, block=1, causal=False, diag_fallback=False)
            return res if out is None else out.copy_(res)
        return sparse_attention(q, kv_contiguous(kc, vc, 1), lists_desc(ids, hkv, counts), causal=False, out=out)

    def selection_lists(self, q, k, offset: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return nsa_select(q, k, self.cfg.block_size, self.selected_blocks, offset=offset)

    def branch_selection(self, q, k, v, offset: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        L.require_cuda(q)
        bs = self.cfg.block_size
        ids, counts = self.selection_lists(q, k, offset)
        self._sel_counts = counts
        if bs == 64 and q.shape[-1] == 128 and q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype:
            res = block_sparse_prefill(q, k, v, ids, counts=counts, rows_per_list=1, causal=False, offset=offset)
            return res if out is None else out.copy_(res)
        if k.stride(3) != 1 or k.stride(2) != k.shape[-1]:
            k, v = k.contiguous(), v.contiguous()
        return sparse_attention(q, kv_contiguous(k, v, bs), lists_desc(ids, q.shape[1], counts), causal=False,
                                out=out)

    def branch_window(self, q, k, v, offset: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        L.require_cuda(q)
        b, hq, tq, _ = q.shape
        hkv, tk = k.shape[1], k.shape[2]
        w = self.cfg.window_size
        n_span = -(-max(w, 1) // 64) + 2  # key blocks a 64-query block's windows can touch
        if (w > 0 and q.shape[-1] == 128 and q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype
                and n_span <= 64):
            # tensor cores: per 64-query block the key blocks of [first - w + 1, last], each
            # row cut to its own window by the kernel
            n_qb, n_kb = -(-tq // 64), -(-tk // 64)
            first = offset + torch.arange(n_qb, device=q.device) * 64
            last = torch.clamp(first + 63, max=offset + tq - 1)
            lo = torch.clamp((first - w + 1).div(64, rounding_mode="floor"), min=0)
            hi = torch.clamp(last.div(64, rounding_mode="floor"), max=n_kb - 1)
            ids = lo[:, None] + torch.arange(n_span, device=q.device)
            ids = torch.where(ids <= hi[:, None], ids, torch.full_like(ids, -1)).to(torch.int32)
            res = block_sparse_prefill(q, k, v, ids.view(1, 1, n_qb, n_span).expand(b, hq, n_qb, n_span),
                                       rows_per_list=64, causal=True, window=w, offset=offset)
            return res if out is None else out.copy_(res)
        if _token_kernel_ok(q, k):
            none = torch.full((b, hkv, 1), -1, dtype=torch.int32, device=q.device)
            res = token_sparse_attention(q, k, v, none, block=1, window=w, causal=True, offset=offset,
                                         diag_fallback=False)
            return res if out is None else out.copy_(res)
        pos = torch.arange(tq, device=q.device) + offset
        wk = (pos - w + 1)[:, None] + torch.arange(max(w, 1), device=q.device)
        ok = (wk >= 0) & (wk <= pos[:, None]) & (wk < tk) & (w > 0)
        wk = torch.where(ok, wk, torch.full_like(wk, -1)).to(torch.int32).view(1, 1, tq, -1)
        wk = wk.expand(b, hkv, tq, wk.shape[-1]).contiguous()
        if k.stride(3) != 1 or k.stride(2) != k.shape[-1]:
            k, v = k.contiguous(), v.contiguous()
        return sparse_attention(q, kv_contiguous(k, v, 1), lists_desc(wk, hkv), causal=False, out=out)

    def _gate_weights(self, dtype, device) -> torch.Tensor:
        if self.gate_mode == "uniform":
            return torch.full((self.cfg.n_heads, 3), 1.0 / 3.0, device=device, dtype=torch.float32)
        g = torch.sigmoid(self.gates.detach().to(device, dtype).float())
        return g / g.sum(-1, keepdim=True).clamp_min(1e-9)

    def _branch_outputs(self, q, k, v, offset: int) -> torch.Tensor:
        """``(3, B, H, T_q, D)`` fp32: compression, selection and window outputs."""
        outs = torch.empty(3, *q.shape, dtype=torch.float32, device=q.device)
        self.branch_compression(q, k, v, offset, out=outs[0])
        self.branch_selection(q, k, v, offset, out=outs[1])
        self.branch_window(q, k, v, offset, out=outs[2])
        return outs

    # -- combination -----------------------------------------------------------------
    def attend(self, q: torch.Tensor, state: Dict[str, Any], offset: int = 0) -> torch.Tensor:
        L.require_cuda(q)
        outs = self._branch_outputs(q, state["k"], state["v"], offset)
        g = self._gate_weights(q.dtype, q.device)
        # three gated terms per head, elementwise (no library GEMV for a 3-term sum)
        gt = g.t()[:, None, :, None, None]  # (3, 1, H, 1, 1)
        mixed = (outs[0] * gt[0] + outs[1] * gt[1]) + outs[2] * gt[2]
        return mixed.to(q.dtype)

    def stats(self) -> Dict[str, float]:
        out = {"reads_per_query": float(self.cfg.window_size + self.selected_blocks * self.cfg.block_size)}
        if self._sel_counts is not None:
            out["selected_blocks_per_query"] = float(self._sel_counts.double().mean())
        return out

    # -- budgets and costs (NSAAttention formulas, native_sparse.py:122-142) -------------
    def read_budget(self, seq_len: int, batch: int = 1) -> float:
        compressed = (seq_len + self.compress - 1) // self.compress
        return float(min(seq_len, self.cfg.window_size + self.selected_blocks * self.cfg.block_size + compressed))

    def memory_bytes(self, seq_len: int, batch: int = 1) -> int:
        return int(batch * self.cfg.n_kv_heads * seq_len * self.cfg.head_dim * 2 * 2)

    def flops(self, seq_len: int, batch: int = 1) -> int:
        h, d = self.cfg.n_heads, self.cfg.head_dim
        compressed = (seq_len + self.compress - 1) // self.compress
        reads = self.cfg.window_size + self.selected_blocks * self.cfg.block_size + compressed
        return int(2 * 2 * batch * h * seq_len * min(seq_len, reads) * d)

    # -- training the gates (native_sparse.py:145-170) -----------------------------------
    def fit_gates(self, q, k, v, steps: int = 200, lr: float = 0.05) -> float:
        """Learn the branch weights that best reproduce causal dense attention.  The
        branch outputs do not depend on the gates, so they are computed once by the
        kernels; the Adam steps run on the (H, 3) gate parameters alone."""
        L.require_cuda(q)
        b, hq, t, d = q.shape
        with torch.no_grad():
            page = 64
            n_pages = -(-k.shape[2] // page)
            kk, vv = k.contiguous(), v.contiguous()
            ids = torch.arange(n_pages, dtype=torch.int32, device=q.device).view(1, 1, n_pages)
            ids = ids.expand(b, k.shape[1], n_pages)
            target = sparse_attention(q, kv_contiguous(kk, vv, page), lists_desc(ids, k.shape[1]), causal=True,
                                      offset=k.shape[2] - t, out=torch.empty(q.shape, dtype=torch.float32,
                                                                              device=q.device))
            outs = self._branch_outputs(q, k, v, 0).to(q.dtype)
            target = target.to(q.dtype)
        gates = self.gates
        if gates.device != q.device:
            gates.data = gates.data.to(q.device)
        opt = torch.optim.Adam([gates], lr=lr)
        loss_value = float("nan")
        for _ in range(steps):
            opt.zero_grad()
            gw = torch.sigmoid(gates).to(q.dtype)
            gw = gw / gw.sum(-1, keepdim=True).clamp_min(1e-9)
            mixed = (gw[:, 0].view(1, -1, 1, 1) * outs[0] + gw[:, 1].view(1, -1, 1, 1) * outs[1]
                     + gw[:, 2].view(1, -1, 1, 1) * outs[2])
            loss = torch.nn.functional.mse_loss(mixed, target)
            loss.backward()
            opt.step()
            loss_value = float(loss.detach())
        self.gate_mode = "learned"
        return loss_value
