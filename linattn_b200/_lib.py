"""ctypes binding of the C ABI in ``include/linattn_b200.h``.

The product path has no fallback: if ``liblinattn_b200.so`` is missing or the
tensors are not on a CUDA device, the call raises.  Argument errors map to
``ValueError`` (as the reference's operators raise, e.g.
``src/linattn/kernels/triton/block_sparse.py:54-55``), unsupported shapes/dtypes
to ``NotImplementedError`` and CUDA failures to ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "_native" / "liblinattn_b200.so"

F32, F16, BF16, FP8E4M3, I32, I64 = 0, 1, 2, 3, 4, 5
DEV_BAD_ID, DEV_TIMEOUT, DEV_OVERFLOW = 1, 2, 4

_DTYPES = {
    torch.float32: F32,
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float8_e4m3fn: FP8E4M3,
    torch.uint8: FP8E4M3,  # raw e4m3 codes
    torch.int32: I32,
    torch.int64: I64,
}

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_vp = ctypes.c_void_p


class KV(ctypes.Structure):
    _fields_ = [
        ("k", c_vp), ("v", c_vp),
        ("stride_b", c_i64), ("stride_page", c_i64), ("stride_head", c_i64),
        ("page_table", c_vp), ("page_table_stride", c_i64), ("num_phys_pages", c_i64),
        ("k_scale", c_vp), ("v_scale", c_vp), ("scale_stride_page", c_i64), ("scale_stride_head", c_i64),
        ("seq_lens", c_vp), ("seq_len", c_i64),
        ("dtype", c_i32), ("page_size", c_i32), ("head_dim", c_i32), ("n_kv_heads", c_i32),
        ("total_rows", c_i64),
    ]


def rows_addressable(t: torch.Tensor, head_dim: int) -> int:
    """D-element rows reachable from ``t.data_ptr()`` to the end of its storage."""
    nbytes = t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()
    return nbytes // (head_dim * t.element_size())


class Meta(ctypes.Structure):
    _fields_ = [
        ("mins", c_vp), ("maxs", c_vp),
        ("stride_b", c_i64), ("stride_page", c_i64), ("stride_head", c_i64),
        ("page_table", c_vp), ("page_table_stride", c_i64), ("num_phys_pages", c_i64),
        ("dtype", c_i32), ("n_heads", c_i32),
    ]


class Lists(ctypes.Structure):
    _fields_ = [
        ("ids", c_vp), ("ids_dtype", c_i32), ("n_heads", c_i32),
        ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64), ("max_len", c_i64),
        ("counts", c_vp), ("cstride_b", c_i64), ("cstride_h", c_i64), ("cstride_t", c_i64),
    ]


_LIB: Optional[ctypes.CDLL] = None
_LOCK = threading.Lock()


def _declare(lib: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    lib.linattn_last_error.restype = ctypes.c_char_p
    lib.linattn_version.restype = ctypes.c_int
    lib.linattn_page_bounds.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, c_i64, P(c_i64), c_i64, c_vp, c_vp, c_vp]
    lib.linattn_paged_page_bounds.argtypes = [P(KV), c_i64, c_vp, c_i64, P(Meta), c_vp, c_vp]
    lib.linattn_paged_append.argtypes = [P(KV), P(Meta), c_i64, c_vp, c_vp, c_i32, P(c_i64), c_i64, c_vp, c_vp,
                                         c_vp]
    lib.linattn_quest_scores.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, c_i64, P(c_i64), P(Meta), c_i64, c_i64,
                                         c_i64, c_i32, c_vp, c_vp, c_vp, c_vp]
    lib.linattn_page_topk.argtypes = [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
                                      c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp]
    lib.linattn_sparse_attention.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), P(KV), P(Lists), c_i32,
                                             c_i64, ctypes.c_float, c_vp, P(c_i64), c_vp, c_i32, c_vp, c_i64, c_vp,
                                             c_vp]
    lib.linattn_sparse_attention_out.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), P(KV), P(Lists), c_i32,
                                                 c_i64, ctypes.c_float, c_vp, c_i32, P(c_i64), c_vp, c_i32, c_vp,
                                                 c_i64, c_vp, c_vp]
    lib.linattn_sparse_attention_out.restype = ctypes.c_int
    lib.linattn_sparse_attention_workspace.argtypes = [c_i64, c_i64, c_i64, c_i64, c_i32]
    lib.linattn_sparse_attention_workspace.restype = c_i64
    lib.linattn_lse_combine.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, c_vp, c_vp]
    lib.linattn_sparse_attention_noalloc.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), P(KV), P(Lists),
                                                     c_i32, c_i64, ctypes.c_float, c_vp, P(c_i64), c_vp, c_i32,
                                                     c_vp, c_vp]
    lib.linattn_sparse_attention_noalloc.restype = ctypes.c_int
    lib.linattn_sparse_attention_noalloc_limit.restype = c_i64
    lib.linattn_quest_decode_select.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), c_vp, c_i32, c_i64, c_i64,
                                                c_vp, c_vp, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_i64,
                                                c_vp, c_vp, c_vp]
    lib.linattn_quest_decode_select.restype = ctypes.c_int
    lib.linattn_indexer_scores.argtypes = [c_vp, c_i32, P(c_i64), c_vp, c_i32, P(c_i64), c_vp, c_i64, c_i64, c_vp,
                                           c_i32, P(c_i64), c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_i64,
                                           c_i64, c_i64, c_vp, c_i64, c_vp, c_vp]
    lib.linattn_row_topk.argtypes = [c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp,
                                     c_vp, c_vp, c_i64, c_i64, c_vp]
    lib.linattn_token_attention.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), c_vp, c_vp, c_vp, c_i64, c_i64,
                                            c_i64, P(c_i64), P(Lists), c_i64, c_i64, c_i64, c_i32, c_i64,
                                            ctypes.c_float, c_i32, c_vp, P(c_i64), c_vp, c_vp, c_vp, c_vp]
    lib.linattn_block_mean.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, c_i64, P(c_i64), c_i64, c_vp, c_vp]
    lib.linattn_csa2_pool_quant.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, c_i64, P(c_i64), c_i64, c_i32, c_i32,
                                            c_vp, c_vp]
    lib.linattn_merge_block_lists.argtypes = [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32,
                                              c_vp, c_i64, c_vp, c_vp]
    lib.linattn_block_sparse_prefill.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                                 c_vp, c_vp, P(c_i64), c_i64, c_i64, P(c_i64), c_i64, c_i32, c_i64,
                                                 c_i64, ctypes.c_float, c_vp, P(c_i64), c_vp, c_vp, c_vp, c_vp, c_vp]
    lib.linattn_prefill_v_to_f16.argtypes = [c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]
    lib.linattn_read_bandwidth.argtypes = [c_vp, c_i64, c_i32, c_vp, c_i64, c_vp]
    lib.linattn_block_score_topk.argtypes = [c_vp, c_i32, P(c_i64), c_vp, c_i32, P(c_i64), c_i64, c_i64, c_i64,
                                             c_i64, c_i64, c_i64, ctypes.c_float, c_i64, c_i64, c_i64, c_i64, c_i64,
                                             c_i64, c_i64, c_i64, c_i32, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp]
    lib.linattn_shard_merge.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64,
                                        c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp]
    lib.linattn_quest_decode_candidates.argtypes = [c_vp, c_i32, c_i64, c_i64, c_i64, P(c_i64), c_vp, c_i32, c_i64,
                                                    c_i64, c_vp, c_i64, c_i32, c_i32, c_i64, c_vp, c_vp, c_vp, c_i64,
                                                    c_vp, c_vp, c_vp]
    lib.linattn_lse_combine_strided.argtypes = [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i32, c_vp, c_vp]
    for name in ("linattn_read_bandwidth", "linattn_block_score_topk", "linattn_shard_merge", "linattn_quest_decode_candidates", "linattn_lse_combine_strided", "linattn_block_sparse_prefill", "linattn_prefill_v_to_f16", "linattn_block_mean", "linattn_csa2_pool_quant", "linattn_merge_block_lists", "linattn_token_attention", "linattn_indexer_scores", "linattn_row_topk", "linattn_page_bounds", "linattn_paged_page_bounds", "linattn_paged_append", "linattn_quest_scores", "linattn_page_topk",
                 "linattn_sparse_attention", "linattn_lse_combine", "linattn_lse_combine_strided"):
        getattr(lib, name).restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """The loaded CUDA library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"linattn_b200 CUDA library not found at {LIB_PATH}; build it with "
                        "`python -m linattn_b200.build` (there is no CPU fallback)")
                handle = ctypes.CDLL(str(LIB_PATH))
                _declare(handle)
                _LIB = handle
    return _LIB


def check(rc: int) -> None:
    if rc == 0:
        return
    msg = (lib().linattn_last_error() or b"").decode()
    if rc == 1:
        raise ValueError(msg)
    if rc == 2:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise NotImplementedError(f"dtype {t.dtype} is not supported by linattn_b200") from None


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def strides4(t: torch.Tensor):
    return (c_i64 * 4)(*t.stride())


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("linattn_b200 operators need CUDA tensors (there is no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


_STATUS: dict = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels OR their LINATTN_DEV_* bits into."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _STATUS.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _STATUS[key] = buf
    return buf


def read_status(device: torch.device, reset: bool = True) -> int:
    """Synchronise and return the device status bits (0 = clean)."""
    buf = status_word(device)
    val = int(buf.item())
    if reset and val:
        buf.zero_()
    return val


def check_status(device: torch.device) -> None:
    bits = read_status(device)
    if bits:
        names = [n for b, n in ((DEV_BAD_ID, "page id outside the page table"), (DEV_TIMEOUT, "bounded wait gave up"),
                                (DEV_OVERFLOW, "union list overflow")) if bits & b]
        raise RuntimeError("linattn_b200 device status: " + ", ".join(names))


def strict() -> bool:
    """When LINATTN_B200_STRICT=1 every operator synchronises and checks the status word."""
    return os.environ.get("LINATTN_B200_STRICT", "0") == "1"
