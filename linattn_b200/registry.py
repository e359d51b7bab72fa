"""The ``cuda_<variant>`` backend slot of the reference registry.

The reference builds backend-native variants by name through ``KERNEL_VARIANTS``
(``<backend>_<variant>``, ``src/linattn/registry.py:139-146``) and ``build``
(``registry.py:225-236``), today only for ``mlx_``.  This module provides the same
API for the CUDA backend: a reference registry dispatches a ``cuda_*`` name here by
calling ``build_cuda(name, cfg)`` from its ``build`` when the prefix matches.
"""

from __future__ import annotations

from typing import Any, Dict, List

from linattn_b200.core import AttentionVariant
from linattn_b200.csa2 import CudaCSA2Attention
from linattn_b200.nsa import CudaNSAAttention
from linattn_b200.variants import CUDA_SUPPORTED, CudaDSAAttention, CudaQuestAttention

__all__ = ["KERNEL_VARIANTS", "build", "build_cuda", "list_kernel_variants", "describe_kernel"]

_CLASSES = {"quest": CudaQuestAttention, "dsa": CudaDSAAttention, "csa2": CudaCSA2Attention, "nsa": CudaNSAAttention}

KERNEL_VARIANTS: Dict[str, str] = {f"cuda_{name}": name for name in CUDA_SUPPORTED}


def build_cuda(variant: str, cfg=None, **kw: Any) -> AttentionVariant:
    """Factory mirroring ``build_mlx`` (``src/linattn/kernels/mlx/adapter.py:105-107``)."""
    if variant not in _CLASSES:
        raise KeyError(f"cuda backend supports {sorted(_CLASSES)}, not {variant!r}")
    return _CLASSES[variant](cfg, **kw)


def build(name: str, cfg=None, **kw: Any) -> AttentionVariant:
    """Instantiate a ``cuda_<variant>`` by name (``registry.py:225-236`` semantics)."""
    if name in KERNEL_VARIANTS:
        backend, _, base = name.partition("_")
        return build_cuda(base, cfg, **kw)
    raise KeyError(f"unknown variant {name!r}; known: {sorted(KERNEL_VARIANTS)}")


def list_kernel_variants() -> List[str]:
    return list(KERNEL_VARIANTS)


def describe_kernel(name: str) -> Dict[str, Any]:
    """Metadata like ``describe_kernel`` (``registry.py:298-310``)."""
    if name not in KERNEL_VARIANTS:
        raise KeyError(f"unknown kernel variant {name!r}; known: {sorted(KERNEL_VARIANTS)}")
    base = KERNEL_VARIANTS[name]
    cls = _CLASSES[base]
    return {"name": name, "class": "cuda_forward", "family": "cuda", "reference": base,
            "citation": getattr(cls, "paper", ())}
