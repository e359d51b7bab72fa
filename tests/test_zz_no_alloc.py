"""The allocation-free entry point ``linattn_sparse_attention_noalloc``.

Some callers cannot allocate device memory where they run attention: an engine that
owns all of HBM through its own pool and forbids side allocations, or a
latency-critical path that cannot take cudaMalloc's implicit device
synchronisation.  For them the library keeps the split-KV scratch in a fixed 64 MiB
device array of its own.  These tests call it through the C ABI and check it
against the allocating entry point ``linattn_sparse_attention`` (caller-provided
workspace), bit for bit, on two calls in a row, and that an oversized request is refused.  This
file is collected last so a failure here never hides the rest of the suite.
"""

from __future__ import annotations

import pytest
import torch

from linattn_b200 import _lib as L
from linattn_b200.block_sparse import kv_contiguous, lists_desc

pytestmark = pytest.mark.gpu

def _case(seed, cuda, b=2):
    gen = torch.Generator().manual_seed(seed)
    hq, hkv, d, bs, t = 8, 2, 128, 64, 64 * 40
    q = torch.randn(b, hq, 1, d, generator=gen).to(torch.bfloat16).to(cuda)
    k = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16).to(cuda)
    v = torch.randn(b, hkv, t, d, generator=gen).to(torch.bfloat16).to(cuda)
    ids = torch.randperm(40, generator=gen)[:23].to(torch.int32).view(1, 1, 23).expand(b, hkv, 23).contiguous()
    return q, k, v, ids.to(cuda), bs


def _call(fn_name, q, k, v, ids, bs, n_splits, workspace=None):
    lib = L.lib()
    kv = kv_contiguous(k, v, bs)
    lists = lists_desc(ids, k.shape[1])
    out = torch.empty_like(q)
    b, hq, tq, d = q.shape
    status = L.status_word(q.device)
    stream = L.stream_of(q)
    if fn_name == "alloc":
        need = lib.linattn_sparse_attention_workspace(b, hq, tq, d, n_splits)
        rc = lib.linattn_sparse_attention(q.data_ptr(), L.dtype_code(q), b, hq, tq, L.strides4(q), kv, lists, 0, 0,
                                          d ** -0.5, out.data_ptr(), L.strides4(out), None, n_splits,
                                          workspace.data_ptr(), need, status.data_ptr(), stream)
    else:
        rc = lib.linattn_sparse_attention_noalloc(q.data_ptr(), L.dtype_code(q), b, hq, tq, L.strides4(q), kv,
                                                  lists, 0, 0, d ** -0.5, out.data_ptr(), L.strides4(out), None,
                                                  n_splits, status.data_ptr(), stream)
    return rc, out


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    # Two calls in a row on different inputs; the second has fewer sequences and fewer
    # splits than the first, so partials the first call left in the shared array
    # would be read by a second call that failed to overwrite them.  Both entry points
    # run the same kernels with the same split count: the outputs must be identical.
    for call, (seed, b, n_splits) in enumerate(((11, 2, 4), (12, 1, 2))):
        q, k, v, ids, bs = _case(seed, cuda, b)
        b, hq, tq, d = q.shape
        need = L.lib().linattn_sparse_attention_workspace(b, hq, tq, d, n_splits)
        ws = torch.empty((need + 3) // 4, dtype=torch.float32, device=cuda)
        rc_a, ref = _call("alloc", q, k, v, ids, bs, n_splits, ws)
        assert rc_a == 0, L.lib().linattn_last_error()
        rc_n, got = _call("noalloc", q, k, v, ids, bs, n_splits)
        assert rc_n == 0, L.lib().linattn_last_error()
        torch.cuda.synchronize()
        assert L.read_status(cuda) == 0
        assert torch.equal(got, ref), f"call {call}: max err {(got.float() - ref.float()).abs().max().item()}"


def test_noalloc_rejects_oversized_scratch(cuda):
    q, k, v, ids, bs = _case(13, cuda)
    limit = L.lib().linattn_sparse_attention_noalloc_limit()
    b, hq, tq, d = q.shape
    ws = L.lib().linattn_sparse_attention_workspace
    per_split = ws(b, hq, tq, d, 3) - ws(b, hq, tq, d, 2)
    too_many = int(limit // per_split) + 2
    assert ws(b, hq, tq, d, too_many) > limit
    rc, _ = _call("noalloc", q, k, v, ids, bs, too_many)
    assert rc == 1
    assert b"limit" in L.lib().linattn_last_error()
