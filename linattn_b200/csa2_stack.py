"""CSA2 cross-layer KV reuse on the sm_100a kernels (``src/linattn/kv/reuse.py``,
``src/linattn/kv/csa2.py``).

``CrossLayerPlan`` partitions layers into groups that share one stored KV copy (the
first layer of each group is the representative).  ``CSA2Stack.run`` runs one
``CudaCSA2Attention`` layer per layer with every layer of a group reading the
representative's K / V; the pooled, quantised copy of that K / V is computed ONCE per
group by ``csa2_pool_quant`` and handed to each layer (the reference recomputes it in
every layer's ``forward``; the values are identical), which is the point of sharing:
one stored copy, one codec pass.  ``compare_share`` measures the divergence that
sharing and low precision cost, as ``compare_share`` in the reference does.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Dict, List, Sequence, Tuple

import torch

from linattn_b200.core import AttnConfig
from linattn_b200.csa2 import CudaCSA2Attention

__all__ = ["CrossLayerPlan", "share_layers", "CSA2StackConfig", "CSA2Stack", "compare_share", "csa2_stack_bytes",
           "csa2_stack_describe"]


@dataclass(frozen=True)
class CrossLayerPlan:
    """Layers ``0 .. n_layers-1`` in consecutive groups of ``group_size``
    (``reuse.py:26-77``)."""

    n_layers: int = 61
    group_size: int = 4

    def __post_init__(self) -> None:
        if self.n_layers < 1:
            raise ValueError("n_layers must be >= 1")
        if self.group_size < 1:
            raise ValueError("group_size must be >= 1")

    @property
    def groups(self) -> List[List[int]]:
        return [list(range(s, min(s + self.group_size, self.n_layers))) for s in range(0, self.n_layers,
                                                                                       self.group_size)]

    @property
    def stored_layers(self) -> List[int]:
        return [g[0] for g in self.groups]

    @property
    def copies(self) -> int:
        return -(-self.n_layers // self.group_size)

    @property
    def bytes_multiplier(self) -> float:
        return self.copies / self.n_layers

    def representative(self, layer: int) -> int:
        if not 0 <= layer < self.n_layers:
            raise IndexError(f"layer {layer} out of range")
        return (layer // self.group_size) * self.group_size

    def is_full(self, layer: int) -> bool:
        return self.representative(layer) == layer

    def as_dict(self) -> Dict[str, object]:
        return {"n_layers": self.n_layers, "group_size": self.group_size, "copies": self.copies,
                "bytes_multiplier": self.bytes_multiplier}


def share_layers(layers: Sequence, plan: CrossLayerPlan) -> Tuple[Dict[int, object], Dict[int, int]]:
    """``(stored, mapping)``: the representatives' entries and, per layer, the
    representative it reads (``reuse.py:80-88``)."""
    if len(layers) != plan.n_layers:
        raise ValueError(f"expected {plan.n_layers} layers, got {len(layers)}")
    stored = {layer: layers[layer] for layer in plan.stored_layers}
    return stored, {layer: plan.representative(layer) for layer in range(plan.n_layers)}


@dataclass
class CSA2StackConfig:
    """Same fields and defaults as the reference's ``CSA2StackConfig`` (``kv/csa2.py:38-48``)."""

    n_layers: int = 8
    layer_group: int = 4
    compress_ratio: int = 32
    bits: int = 4
    quant_group: int = 32
    topk_groups: int = 8
    window: int = 128
    share: bool = True
    seed: int = 0


def csa2_stack_bytes(cfg: CSA2StackConfig, attn: AttnConfig, seq_len: int, n_layers: int, batch: int = 1) -> float:
    """Stored bytes for one request (``KVSpec.bytes_for``, ``kv/format.py``): the K and V
    values of a token, pooled by the compression ratio, quantised with one fp16 scale per
    ``quant_group`` values (2 bytes per value at 16 bits), one copy per layer group."""
    values = (2 * attn.n_kv_heads * attn.head_dim / cfg.compress_ratio) * seq_len
    n = max(1, int(math.ceil(values)))
    per_copy = n * 2.0 if cfg.bits >= 16 else n * cfg.bits / 8.0 + math.ceil(n / cfg.quant_group) * 2.0
    group = cfg.layer_group if cfg.share else 1
    return per_copy * max(1, math.ceil(n_layers / group)) * batch


def csa2_stack_describe(cfg: CSA2StackConfig, attn: AttnConfig) -> str:
    """``KVSpec.describe`` of the stack's storage (``kv/format.py``)."""
    parts = [f"{2 * attn.n_kv_heads * attn.head_dim:g} values/token"]
    if cfg.compress_ratio > 1:
        parts.append(f"pooled x{cfg.compress_ratio}")
    parts.append(f"fp{cfg.bits}" if cfg.bits < 16 else "fp16")
    group = cfg.layer_group if cfg.share else 1
    if group > 1:
        parts.append(f"shared over {group} layers")
    return ", ".join(parts)


class CSA2Stack:
    """``CSA2Stack`` (``kv/csa2.py:60-99``) on the CUDA layer."""

    def __init__(self, cfg: CSA2StackConfig, attn: AttnConfig):
        self.cfg = cfg
        self.attn_cfg = attn
        self.plan = CrossLayerPlan(n_layers=cfg.n_layers, group_size=cfg.layer_group)
        extras = {"compress_ratio": cfg.compress_ratio, "bits": cfg.bits, "quant_group": cfg.quant_group,
                  "topk_groups": cfg.topk_groups, "window": cfg.window,
                  "cross_layer_group": cfg.layer_group if cfg.share else 1}
        self.layer = CudaCSA2Attention(attn.with_(extras=extras))

    def run(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Dict[str, object]:
        """``q, k, v``: ``(n_layers, B, H, T, D)`` (K / V with the kv heads)."""
        n_layers = q.shape[0]
        if n_layers != self.cfg.n_layers:
            raise ValueError(f"expected {self.cfg.n_layers} layers, got {n_layers}")
        outs: List[torch.Tensor] = []
        reads: List[float] = []
        cached: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        # the reference runs each layer's forward with chunk = q.shape[2] (the head axis of
        # these 5-D inputs) and keeps the last chunk's statistic; the outputs do not depend
        # on the chunking, so all queries attend at once and the statistic is taken over
        # the same last rows
        t, c = q.shape[-2], q.shape[2]
        last = slice(((t - 1) // c) * c, t)
        with torch.no_grad():
            for layer in range(n_layers):
                src = self.plan.representative(layer) if self.cfg.share else layer
                if src not in cached:  # one codec pass per stored copy
                    cached = {src: self.layer.compressed_kv(k[src], v[src])}
                outs.append(self.layer.attend_kv(q[layer], k[src], v[src], offset=0, compressed=cached[src]))
                reads.append(self.layer.stats(rows=last)["reads_per_query"])
        seq = q.shape[-2]
        per_seq_bytes = csa2_stack_bytes(self.cfg, self.attn_cfg, seq, n_layers) / max(1, q.shape[1])
        return {"out": torch.stack(outs), "reads_per_query": sum(reads) / len(reads),
                "copies": self.plan.copies if self.cfg.share else n_layers, "bytes_per_token": per_seq_bytes / seq,
                "spec": csa2_stack_describe(self.cfg, self.attn_cfg)}


def compare_share(cfg: CSA2StackConfig, attn: AttnConfig, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  baseline_bits: int = 16) -> Dict[str, float]:
    """Shared stack vs the per-layer stack vs a per-layer stack at ``baseline_bits``
    (``kv/csa2.py:102-131``)."""
    per_layer_cfg = replace(cfg, share=False)
    ref = CSA2Stack(replace(per_layer_cfg, bits=baseline_bits), attn).run(q, k, v)
    base = CSA2Stack(per_layer_cfg, attn).run(q, k, v)
    sh = CSA2Stack(cfg, attn).run(q, k, v)

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))

    return {"divergence_shared_vs_ref": rel(sh["out"], ref["out"]),
            "divergence_unshared_vs_ref": rel(base["out"], ref["out"]),
            "sharing_delta": rel(sh["out"], base["out"]),
            "bytes_per_token_shared": sh["bytes_per_token"], "bytes_per_token_unshared": base["bytes_per_token"],
            "copies_shared": sh["copies"], "copies_unshared": base["copies"],
            "reads_per_query": sh["reads_per_query"]}
