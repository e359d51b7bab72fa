"""The C ABI: the library loads, exports every entry point ``include/*.h`` declares,
and rejects bad arguments on the host (no GPU work, so these run on CPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from linattn_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(linattn_\w+)\s*\(", text, flags=re.M))
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    assert {"linattn_page_bounds", "linattn_quest_scores", "linattn_page_topk", "linattn_sparse_attention",
            "linattn_lse_combine", "linattn_paged_page_bounds"} <= names


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for name in _declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert lib.linattn_version() >= 1


def test_host_validation_without_gpu():
    lib = L.lib()
    # n_pages outside the supported range: rejected before any launch
    rc = lib.linattn_page_topk(None, 1, 1, 1, 0, 1, None, None, None, 1, None, None, 0, None, 1, 0, None, 0, None,
                               None)
    assert rc == 1  # scores NULL -> EINVAL
    rc = lib.linattn_page_topk(ctypes.c_void_p(16), 1, 1, 1, 0, 1, None, None, None, 1, None, None, 0, None, 1, 0,
                               None, 0, None, None)
    assert rc == 2 and b"n_pages" in lib.linattn_last_error()
    with pytest.raises(NotImplementedError):
        L.check(rc)
    kv = L.KV()
    kv.dtype = 99
    rc = lib.linattn_sparse_attention(ctypes.c_void_p(16), 2, 1, 1, 1, (L.c_i64 * 4)(0, 0, 0, 1), kv, L.Lists(), 0,
                                      0, 1.0, ctypes.c_void_p(16), (L.c_i64 * 4)(0, 0, 0, 1), None, 1, None, 0, None,
                                      None)
    assert rc == 2 and b"kv dtype" in lib.linattn_last_error()
    assert lib.linattn_sparse_attention_workspace(2, 8, 1, 128, 1) == 256
    assert lib.linattn_sparse_attention_workspace(2, 8, 1, 128, 4) == 256 + 4 * 2 * 8 * 129 * 4


def test_operators_refuse_cpu_tensors():
    import torch

    from linattn_b200 import block_sparse_attention, page_bounds

    with pytest.raises(ValueError, match="CUDA"):
        page_bounds(torch.zeros(1, 1, 8, 8), 4)
    with pytest.raises(ValueError, match="block_size"):
        block_sparse_attention(torch.zeros(1, 1, 1, 8), torch.zeros(1, 1, 8, 8), torch.zeros(1, 1, 8, 8),
                               torch.zeros(1, 1, 1, dtype=torch.long))
    with pytest.raises(ValueError, match="backend"):
        block_sparse_attention(torch.zeros(1, 1, 1, 8), torch.zeros(1, 1, 8, 8), torch.zeros(1, 1, 8, 8),
                               torch.zeros(1, 1, 1, dtype=torch.long), block_size=4, backend="torch")
