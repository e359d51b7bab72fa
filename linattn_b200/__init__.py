"""linattn_b200: the sparse-attention hot path of tongxin/linattn on NVIDIA B200 (sm_100a).

Operators (same names and semantics as ``linattn.kernels.triton.*``):
``page_bounds``, ``page_select``, ``block_sparse_attention``, ``indexer_topk``,
``lse_combine``.
Plugin: ``build("cuda_quest" | "cuda_dsa" | "cuda_csa2" | "cuda_nsa", cfg)`` returns an ``AttentionVariant`` like
``linattn.registry.build``.  Serving path: ``PagedKVCache`` + ``QuestDecoder``.

Every call runs hand-written CUDA in ``_native/liblinattn_b200.so`` through the C
ABI of ``include/linattn_b200.h``; there is no CPU fallback.
"""

from linattn_b200.block_sparse import block_sparse_attention, sparse_attention  # noqa: F401
from linattn_b200.core import AttnConfig, AttentionVariant  # noqa: F401
from linattn_b200.csa2 import CudaCSA2Attention, csa2_pool_quant  # noqa: F401
from linattn_b200.nsa import CudaNSAAttention, nsa_select  # noqa: F401
from linattn_b200.indexer import indexer_scores, indexer_topk, quantize_keys_fp8, row_topk  # noqa: F401
from linattn_b200.merge import lse_combine  # noqa: F401
from linattn_b200.paged import PagedKVCache, QuestDecodeGraph, QuestDecoder  # noqa: F401
from linattn_b200.quest_pages import page_bounds, page_select, quest_select  # noqa: F401
from linattn_b200.registry import KERNEL_VARIANTS, build, build_cuda, describe_kernel, list_kernel_variants  # noqa: F401

__version__ = "0.1.0"
