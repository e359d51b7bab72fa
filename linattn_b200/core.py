"""The variant contract of the reference, restated for the CUDA variants.

``AttnConfig`` has the fields of ``src/linattn/core.py:47-78`` and
``AttentionVariant`` the streaming driver of ``core.py:187-306``:
``forward(q, k, v, state=None, chunk=None) -> (out, state)`` walks the query axis in
chunks, appends each chunk's keys/values (``push_kv``) and calls ``attend`` with the
absolute offset of the chunk.  A reference ``AttnConfig`` instance can be passed
anywhere this one is accepted (only its attributes are read).
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Any, Dict, Optional

import torch

__all__ = ["AttnConfig", "AttentionVariant"]


@dataclass
class AttnConfig:
    n_heads: int = 4
    n_kv_heads: int = 4
    head_dim: int = 64
    block_size: int = 64
    window_size: int = 256
    cache_budget: int = 512
    topk_blocks: int = 4
    topk_tokens: int = 256
    compress_ratio: int = 16
    obs_window: int = 64
    sink_size: int = 4
    stride: int = 8
    threshold: float = 0.9
    dtype: torch.dtype = torch.float32
    seed: int = 0
    extras: Dict[str, Any] = field(default_factory=dict)

    @property
    def group_size(self) -> int:
        return max(1, self.n_heads // self.n_kv_heads)

    def with_(self, **kw: Any) -> "AttnConfig":
        return replace(self, **kw)


class AttentionVariant:
    """Chunked streaming driver (``src/linattn/core.py:187-306``)."""

    name: str = "base"
    family: str = "dense"
    trained: bool = False
    paper: tuple = ()

    def __init__(self, cfg: Optional[Any] = None, **kwargs: Any) -> None:
        self.cfg = cfg if cfg is not None else AttnConfig()
        for key, value in kwargs.items():
            if not hasattr(self.cfg, key):
                raise TypeError(f"{type(self).__name__}: unknown config field {key!r}")
            setattr(self.cfg, key, value)
        if self.cfg.n_heads % self.cfg.n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")

    @property
    def group_size(self) -> int:
        return max(1, self.cfg.n_heads // self.cfg.n_kv_heads)

    def prepare_state(self, batch: int, device, dtype) -> Dict[str, Any]:
        z = torch.zeros(batch, self.cfg.n_kv_heads, 0, self.cfg.head_dim, device=device, dtype=dtype)
        return {"k": z, "v": z.clone(), "pos": 0}

    def push_kv(self, state: Dict[str, Any], k: torch.Tensor, v: torch.Tensor) -> Dict[str, Any]:
        state["k"] = torch.cat([state["k"], k], dim=-2)
        state["v"] = torch.cat([state["v"], v], dim=-2)
        return state

    def attend(self, q: torch.Tensor, state: Dict[str, Any], offset: int = 0) -> torch.Tensor:
        raise NotImplementedError

    def finalize(self, state: Dict[str, Any]) -> Dict[str, Any]:
        return state

    def default_chunk(self) -> int:
        return 256

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, state: Optional[Dict[str, Any]] = None,
                chunk: Optional[int] = None, causal: bool = True, collect_stats: bool = False):
        if q.dim() != 4:
            raise ValueError("q must have shape (B, H, T, D)")
        b, h, t, d = q.shape
        if state is None:
            state = self.prepare_state(b, q.device, q.dtype)
        chunk = chunk or max(1, self.default_chunk())
        outs = []
        pos = state.get("pos", 0)
        stats = [] if collect_stats else None
        for start in range(0, t, chunk):
            stop = min(start + chunk, t)
            state = self.push_kv(state, k[:, :, start:stop], v[:, :, start:stop])
            outs.append(self.attend(q[:, :, start:stop], state, offset=pos + start))
            state = self.finalize(state)
            if stats is not None:
                stats.append(self.stats())
        state["pos"] = pos + t
        out = torch.cat(outs, dim=-2)
        if collect_stats:
            return out, state, stats
        return out, state

    def stats(self) -> Dict[str, float]:
        return {}

    def memory_bytes(self, seq_len: int, batch: int = 1) -> int:
        return batch * self.cfg.n_kv_heads * seq_len * self.cfg.head_dim * 2 * 2

    def flops(self, seq_len: int, batch: int = 1) -> int:
        return int(2 * 2 * batch * self.cfg.n_heads * seq_len * seq_len * self.cfg.head_dim)

    def read_budget(self, seq_len: int, batch: int = 1) -> float:
        return float(seq_len)
