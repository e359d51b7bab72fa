"""The C restatement (oracle/c/oracle.c, the full-size checker and CPU baseline)
agrees with the numpy oracle, and the reference's own C kernel (oracle/_ref) agrees
with both on the paged decode it implements."""

from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "_build" / "liboracle.so"
REF = ROOT / "oracle" / "_ref" / "libdecode_attn.so"


@pytest.fixture(scope="module")
def ora():
    if not LIB.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    lib = ctypes.CDLL(str(LIB))
    lib.oracle_quest_decode.restype = ctypes.c_int
    return lib


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest-even) and return the 16-bit patterns."""
    u = x.astype(np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def _bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("lens", [[640, 640], [640, 200]])
def test_c_oracle_matches_numpy_oracle(ora, lens):
    rng = np.random.default_rng(sum(lens))
    b, hq, hkv, d, p, topk, sink = 2, 8, 2, 64, 16, 6, 1
    max_pages = 40
    n_phys = b * max_pages
    kb = _bf16_bits(rng.standard_normal((n_phys, hkv, p, d)).astype(np.float32))
    vb = _bf16_bits(rng.standard_normal((n_phys, hkv, p, d)).astype(np.float32))
    qb = _bf16_bits(rng.standard_normal((b, hq, d)).astype(np.float32))
    table = rng.permutation(n_phys).astype(np.int32).reshape(b, max_pages)
    lens = np.array(lens, dtype=np.int32)
    kf, vf, qf = _bits_to_f32(kb), _bits_to_f32(vb), _bits_to_f32(qb)
    # metadata per physical page over its valid rows
    mn = np.zeros((n_phys, hkv, d), np.float32)
    mx = np.zeros((n_phys, hkv, d), np.float32)
    for bi in range(b):
        for pg in range((lens[bi] + p - 1) // p):
            ph = table[bi, pg]
            rows = min(p, lens[bi] - pg * p)
            mn[ph] = kf[ph, :, :rows].min(1)
            mx[ph] = kf[ph, :, :rows].max(1)
    mnb, mxb = _bf16_bits(mn), _bf16_bits(mx)  # exact: values came from bf16
    max_union = min(hq // hkv * topk, max_pages)
    out = np.zeros((b, hq, d), np.float32)
    uids = np.zeros((b, hkv, max_union), np.int32)
    ucnt = np.zeros((b, hkv), np.int32)
    P_ = ctypes.c_void_p
    rc = ora.oracle_quest_decode(2, P_(qb.ctypes.data), P_(kb.ctypes.data), P_(vb.ctypes.data),
                                 P_(mnb.ctypes.data), P_(mxb.ctypes.data), P_(table.ctypes.data),
                                 P_(lens.ctypes.data), b, hq, hkv, d, p, max_pages, topk, sink,
                                 ctypes.c_float(1 / math.sqrt(d)), P_(out.ctypes.data), P_(uids.ctypes.data),
                                 P_(ucnt.ctypes.data), max_union, 0, b * hkv)
    assert rc == 0
    # numpy oracle: logical contiguous K for the selection
    for bi in range(b):
        nb = (lens[bi] + p - 1) // p
        mins = mn[table[bi, :nb]].transpose(1, 0, 2)[None]  # (1, Hkv, nb, D)
        maxs = mx[table[bi, :nb]].transpose(1, 0, 2)[None]
        ids, _ = oracle.page_select(qf[bi:bi + 1, :, None], mins, maxs, p, topk, offset=1 << 40, sink_pages=sink)
        union = oracle.gqa_union(ids, nb, hq // hkv)[0, :, 0]
        for kh in range(hkv):
            assert np.array_equal(uids[bi, kh, : ucnt[bi, kh]], np.nonzero(union[kh])[0])
    ref = oracle.paged_sparse_decode(qf, kf, vf, table, lens, uids, ucnt, page_size=p)
    assert np.abs(out - ref).max() < 1e-5


def test_reference_c_kernel_matches_oracle():
    if not REF.exists():
        pytest.skip("reference source not present when oracle/_ref was built")
    lib = ctypes.CDLL(str(REF))
    f32p = ctypes.POINTER(ctypes.c_float)
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib.paged_decode_tiled.argtypes = [f32p, f32p, f32p, i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, f32p]
    rng = np.random.default_rng(0)
    t, d, p = 512, 64, 8
    k = rng.standard_normal((t, d)).astype(np.float32)
    v = rng.standard_normal((t, d)).astype(np.float32)
    q = rng.standard_normal(d).astype(np.float32)
    pages = np.array([0, 5, 17, 63, 40, 9], dtype=np.int32)
    out = np.zeros(d, np.float32)
    lib.paged_decode_tiled(q.ctypes.data_as(f32p), k.ctypes.data_as(f32p), v.ctypes.data_as(f32p),
                           pages.ctypes.data_as(i32p), len(pages), p, d, t, ctypes.c_float(1 / math.sqrt(d)),
                           out.ctypes.data_as(f32p))
    ref = oracle.paged_sparse_decode(q[None, None], k.reshape(t // p, 1, p, d), v.reshape(t // p, 1, p, d),
                                     np.arange(t // p)[None], np.array([t]), pages[None, None],
                                     np.array([[len(pages)]]), page_size=p)
    assert np.abs(out - ref[0, 0]).max() < 2e-4  # tests/test_kernels.py:42 tolerance
