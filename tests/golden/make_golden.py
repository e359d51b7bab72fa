"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Run in the build container, where the reference project is importable from its
source tree (read-only; bytecode writing is disabled so nothing is written there):

    python tests/golden/make_golden.py [--ref /path/to/linattn/checkout]

Each ``.npz`` holds seeded inputs and the outputs of the reference functions named
in its ``fn`` entry.  The fixtures travel with the repository; the GPU box never
needs the reference.  ``tests/test_oracle_golden.py`` pins the CPU oracle to them and
``tests/test_gpu_parity.py`` checks the CUDA library against them.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _import_reference(ref_root: Path):
    sys.dont_write_bytecode = True
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.path.insert(0, str(ref_root / "src"))
    import torch  # noqa: F401

    import linattn  # noqa: F401
    return linattn


def _np(t):
    import torch

    if t.dtype == torch.bool:
        return t.numpy().copy()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.float().numpy().copy()
    return t.detach().numpy().copy()


def make_page_bounds(out):
    import torch
    from linattn.kernels.triton.quest_pages import page_bounds_torch

    torch.manual_seed(0)
    k64 = torch.randn(1, 2, 32, 8, dtype=torch.float64)  # tests/test_kernels.py:98-108 shape
    m64, x64 = page_bounds_torch(k64, 8)
    g = torch.Generator().manual_seed(11)
    k32 = torch.randn(2, 2, 37, 16, generator=g)  # ragged tail page
    m32, x32 = page_bounds_torch(k32, 8)
    np.savez_compressed(out / "page_bounds.npz", fn="page_bounds_torch", k64=_np(k64), min64=_np(m64),
                        max64=_np(x64), k32=_np(k32), min32=_np(m32), max32=_np(x32), page64=8, page32=8)


def make_page_select(out):
    import torch
    from linattn.kernels.triton.quest_pages import page_bounds_torch, page_select_torch

    g = torch.Generator().manual_seed(21)
    b, hq, hkv, t, d, page = 2, 8, 2, 200, 32, 16
    k = torch.randn(b, hkv, t, d, generator=g)
    q = torch.randn(b, hq, 1, d, generator=g)
    from linattn.core import repeat_kv

    # the operator has no GQA axis: metadata is per query head (repeat_kv, as
    # QuestAttention.page_scores does at src/linattn/variants/selection.py:207-208)
    mins, maxs = (repeat_kv(x, hq // hkv) for x in page_bounds_torch(k, page))
    rec = {"fn": "page_select_torch", "q": _np(q), "k": _np(k), "mins": _np(mins), "maxs": _np(maxs),
           "page": page, "offset": t - 1}
    for topk in (1, 4, 13, 40):  # 40 > n_pages (13): k clamps to n_pages
        ids, scores = page_select_torch(q, mins, maxs, page, topk, offset=t - 1)
        rec[f"ids_{topk}"] = _np(ids)
        rec[f"scores_{topk}"] = _np(scores)
    # fp16 inputs, decode at a position inside the sequence (pages after it invisible)
    qh = q.half()
    kh = k.half()
    mh, xh = (repeat_kv(x, hq // hkv) for x in page_bounds_torch(kh, page))
    ids, scores = page_select_torch(qh.float(), mh.float(), xh.float(), page, 5, offset=100)
    rec.update(q16=_np(qh), k16=_np(kh), mins16=_np(mh), maxs16=_np(xh), ids16_5=_np(ids),
               scores16_5=_np(scores), offset16=100)
    np.savez_compressed(out / "page_select.npz", **rec)


def make_topk_ties(out):
    import torch

    g = torch.Generator().manual_seed(5)
    s = torch.randint(0, 6, (4, 64), generator=g).float()  # heavy ties
    s[:, 3] = float("inf")
    s[:, 40:] = float("-inf")
    vals, ids = torch.topk(s, 10, dim=-1)
    np.savez_compressed(out / "topk_ties.npz", fn="torch.topk", scores=_np(s), ids=_np(ids), vals=_np(vals), k=10)


def make_quest_variant(out):
    import torch
    from linattn.core import AttnConfig
    from linattn.harness import structured_inputs
    from linattn.registry import build

    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=32, cache_budget=64,
                     topk_blocks=3, topk_tokens=48, compress_ratio=8, obs_window=16, sink_size=2, stride=4)
    q, k, v = structured_inputs(1, 4, 192, 32, kv_heads=2, seed=1)  # tests/conftest.py:174-177
    q, k, v = q.double(), k.double(), v.double()
    # inputs are float32 draws (exact in float32); outputs stay float64
    rec = {"fn": "QuestAttention", "q": _np(q.float()), "k": _np(k.float()), "v": _np(v.float()), "page": 16,
           "topk": 3}
    for label, extras in (("union", {}), ("nounion", {"gqa_union": False})):
        var = build("quest", cfg.with_(extras=dict(extras)))
        state = var.prepare_state(1, q.device, q.dtype)
        state = var.push_kv(state, k, v)
        rec[f"mask_{label}"] = _np(var.effective_mask(q, state, 0))
        with torch.no_grad():
            o64, _ = build("quest", cfg.with_(extras=dict(extras))).forward(q, k, v, chunk=64)
            o192, _ = build("quest", cfg.with_(extras=dict(extras))).forward(q, k, v, chunk=192)
        rec[f"out64_{label}"] = _np(o64)
        rec[f"out192_{label}"] = _np(o192)
    # decode: one query after a 191-token prefill, union mode
    var = build("quest", cfg)
    with torch.no_grad():
        _, st = var.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
        od, _ = var.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
    rec["out_decode"] = _np(od)
    rec["reads_decode"] = var.stats()["reads_per_query"]
    np.savez_compressed(out / "quest_variant.npz", **rec)


def make_dsa_variant(out):
    import torch
    from linattn.core import AttnConfig
    from linattn.harness import structured_inputs
    from linattn.registry import build

    q, k, v = structured_inputs(1, 4, 192, 32, kv_heads=2, seed=3)
    rec = {"fn": "DSAAttention", "q": _np(q.float()), "k": _np(k.float()), "v": _np(v.float())}
    # token-level (compress_ratio 1) and compressed (CSA, ratio 4) selections
    for label, ratio in (("tok", 1), ("csa", 4)):
        cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=24, topk_tokens=40,
                         compress_ratio=ratio, sink_size=2, seed=5)
        var = build("dsa", cfg)
        state = var.prepare_state(1, q.device, q.dtype)
        state = var.push_kv(state, k, v)
        with torch.no_grad():
            rec[f"mask_{label}"] = _np(var.effective_mask(q, state, 0))
            rec[f"scores_{label}"] = _np(var.indexer_scores(q, k if ratio == 1 else _pool(k, ratio)))
            o64, _ = build("dsa", cfg).forward(q, k, v, chunk=64)
            o192, _ = build("dsa", cfg).forward(q, k, v, chunk=192)
            var2 = build("dsa", cfg)
            var2.forward(q, k, v, chunk=192)
        rec[f"out64_{label}"] = _np(o64)
        rec[f"out192_{label}"] = _np(o192)
        rec[f"reads_{label}"] = var2.stats()["reads_per_query"]
    np.savez_compressed(out / "dsa_variant.npz", **rec)


def _pool(k, m):
    from linattn.core import block_reduce
    return block_reduce(k, m, -2)


def make_block_sparse(out):
    import torch
    from linattn.kernels.triton.block_sparse import block_sparse_attention_torch

    torch.manual_seed(0)
    b, h, t, d, bs = 1, 4, 128, 64, 32  # tests/test_kernels.py:126-138 shape (fp32, CPU)
    q = torch.randn(b, h, t, d)
    k = torch.randn(b, h, t, d)
    v = torch.randn(b, h, t, d)
    ids = torch.randint(0, t // bs, (b, h, t, 2))
    ids[..., 1] = torch.arange(t) // bs
    o1 = block_sparse_attention_torch(q, k, v, ids, block_size=bs)
    g = torch.Generator().manual_seed(3)
    q2 = torch.randn(2, 8, 5, 32, generator=g)
    k2 = torch.randn(2, 2, 100, 32, generator=g)
    v2 = torch.randn(2, 2, 100, 32, generator=g)
    ids2 = torch.tensor([[[0, 6, 3], [2, 6, 5]], [[1, 1, 4], [6, 0, 2]]])  # (B,Hkv,N): tail block 6, a duplicate
    o2 = block_sparse_attention_torch(q2, k2, v2, ids2, block_size=16)
    ids_all = torch.arange(t // bs).view(1, 1, 1, -1).expand(b, h, t, -1)
    o3 = block_sparse_attention_torch(q, k, v, ids_all, block_size=bs)
    np.savez_compressed(out / "block_sparse.npz", fn="block_sparse_attention_torch", q=_np(q), k=_np(k), v=_np(v),
                        ids=_np(ids), out=_np(o1), bs=bs, q2=_np(q2), k2=_np(k2), v2=_np(v2), ids2=_np(ids2),
                        out2=_np(o2), bs2=16, out_all=_np(o3))


def make_indexer(out):
    import torch
    from linattn.kernels.triton.fused_indexer import indexer_topk_torch

    torch.manual_seed(0)
    b, tq, tk, hi, d, kk = 1, 8, 32, 3, 8, 5  # tests/test_kernels.py:86-95
    q_idx = torch.randn(b, tq, hi, d)
    k_idx = torch.randn(b, tq * 0 + tk, hi, d)
    w = torch.rand(b, tq, hi)
    vals, idx = indexer_topk_torch(q_idx, k_idx, w, kk)
    g = torch.Generator().manual_seed(9)
    q2 = torch.randn(2, 16, 4, 16, generator=g)
    k2 = torch.randn(2, 64, 4, 16, generator=g)
    w2 = torch.randn(2, 16, 4, generator=g) / 8
    v2, i2 = indexer_topk_torch(q2, k2, w2, 10)
    np.savez_compressed(out / "indexer.npz", fn="indexer_topk_torch", q=_np(q_idx), k=_np(k_idx), w=_np(w),
                        vals=_np(vals), idx=_np(idx), topk=kk, q2=_np(q2), k2=_np(k2), w2=_np(w2), vals2=_np(v2),
                        idx2=_np(i2), topk2=10)


def make_dense(out):
    import torch
    from linattn.core import dense_attention

    g = torch.Generator().manual_seed(4)
    q = torch.randn(2, 6, 7, 16, generator=g, dtype=torch.float64)
    k = torch.randn(2, 3, 19, 16, generator=g, dtype=torch.float64)
    v = torch.randn(2, 3, 19, 16, generator=g, dtype=torch.float64)
    o_c = dense_attention(q, k, v, causal=True)
    o_n = dense_attention(q, k, v, causal=False)
    np.savez_compressed(out / "dense.npz", fn="dense_attention", q=_np(q), k=_np(k), v=_np(v), out_causal=_np(o_c),
                        out_full=_np(o_n))


def make_block_selectors(out):
    from linattn.core import AttnConfig
    from linattn.harness import structured_inputs
    from linattn.registry import build

    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=32, cache_budget=64,
                     topk_blocks=3, topk_tokens=48, compress_ratio=8, obs_window=16, sink_size=2, stride=4)
    q, k, v = structured_inputs(1, 4, 192, 32, kv_heads=2, seed=1)
    q, k, v = q.double(), k.double(), v.double()
    mi = build("minference", cfg.with_(extras={"pattern": "block_sparse"}))
    mask_mi = mi._block_sparse(q, k, 0)
    moba = build("moba", cfg)
    st = moba.prepare_state(1, q.device, q.dtype)
    st = moba.push_kv(st, k, v)
    mask_moba = moba.select(q, st, 0)
    np.savez_compressed(out / "block_selectors.npz", fn="MInferenceAttention._block_sparse,MoBAAttention.select",
                        q=_np(q.float()), k=_np(k.float()), block=16, topk=3, sink=2, mask_minference=_np(mask_mi),
                        mask_moba=_np(mask_moba))


def make_quant(out):
    import torch
    from linattn.kv.quant import QuantSpec, dequantize, quantize

    g = torch.Generator().manual_seed(8)
    x = torch.randn(4, 96, generator=g) * torch.linspace(0.1, 5, 96)
    spec = QuantSpec(bits=8, group_size=32)
    codes, scales = quantize(x, spec)
    xh = dequantize(codes, scales, spec)
    np.savez_compressed(out / "quant.npz", fn="kv.quant fp8", x=_np(x), codes=codes.view(torch.uint8).numpy().copy(),
                        scales=_np(scales), xhat=_np(xh), group=32)


def make_paged_decode(out):
    import torch
    from linattn.kernels.c_attention import build_library, paged_decode, paged_decode_torch

    g = torch.Generator().manual_seed(2)
    t, dim, page = 512, 64, 8
    k = torch.randn(t, dim, generator=g)
    v = torch.randn(t, dim, generator=g)
    q = torch.randn(dim, generator=g)
    pages = torch.tensor([0, 5, 17, 63, 40, 9])
    ref = paged_decode_torch(q, k, v, pages, page_size=page)
    rec = {"fn": "paged_decode_torch", "q": _np(q), "k": _np(k), "v": _np(v), "pages": _np(pages), "page": page,
           "out": _np(ref)}
    if build_library() is not None:
        o_c, _ = paged_decode(q, k, v, pages, page_size=page, kernel="tiled")
        rec["out_c_tiled"] = _np(o_c)
    np.savez_compressed(out / "paged_decode.npz", **rec)


def make_csa2_variant(out):
    import torch
    from linattn.core import AttnConfig
    from linattn.harness import structured_inputs
    from linattn.registry import build

    rec = {"fn": "CSA2Attention"}
    # codec: compressed_kv of one tensor in bf16 / f16 / f32, ragged tail (T = 50), a
    # partial quantisation group (D = 48), channel scales spread over 60x, and one
    # all-zero (token group, channel group) to reach the 1e-8 scale clamp
    gen = torch.Generator().manual_seed(11)
    dtypes = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
    for d in (48, 128):
        x = torch.randn(1, 2, 50, d, generator=gen) * torch.linspace(0.05, 3.0, d)
        x[0, 1, :12, :32] = 0.0
        rec[f"codec_x_d{d}"] = _np(x)
        for name, dt in dtypes.items():
            for ratio in (3, 4):
                for bits in (4, 8, 16):
                    cfg = AttnConfig(n_heads=2, n_kv_heads=2, head_dim=d,
                                     extras={"compress_ratio": ratio, "bits": bits})
                    kc, _ = build("csa2", cfg).compressed_kv(x.to(dt), x.to(dt))
                    rec[f"codec_{name}_d{d}_m{ratio}_b{bits}"] = _np(kc.float())
    # the variant in float32: chunked prefill (64 / 192) and one decode step
    q, k, v = structured_inputs(1, 4, 192, 32, kv_heads=2, seed=7)
    q, k, v = q.float(), k.float(), v.float()
    rec.update(q=_np(q), k=_np(k), v=_np(v))
    for bits in (4, 8):
        cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, window_size=24, topk_blocks=3, compress_ratio=8,
                         seed=5, extras={"bits": bits})
        var = build("csa2", cfg)
        with torch.no_grad():
            kc, _ = var.compressed_kv(k, v)
            rec[f"scores_b{bits}"] = _np(var.indexer_scores(q, kc))
            rec[f"q_proj_b{bits}"] = _np(var.q_proj.detach())
            for chunk in (64, 192):
                v2 = build("csa2", cfg)
                o, _ = v2.forward(q, k, v, chunk=chunk)
                rec[f"out{chunk}_b{bits}"] = _np(o)
                for key, val in v2.stats().items():
                    rec[f"stats{chunk}_b{bits}_{key}"] = float(val)
            v3 = build("csa2", cfg)
            _, st = v3.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
            od, _ = v3.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
            rec[f"out_decode_b{bits}"] = _np(od)
            rec[f"reads_decode_b{bits}"] = float(v3.stats()["reads_per_query"])
    # accounting (read_budget / memory_bytes / selection_flops) for a few settings
    acct = []
    for extras in ({}, {"bits": 8, "cross_layer_group": 2}, {"bits": 16, "compress_ratio": 4, "topk_groups": 9}):
        var = build("csa2", AttnConfig(n_heads=8, n_kv_heads=2, head_dim=64, extras=dict(extras)))
        for n in (5, 100, 4096):
            acct.append([var.read_budget(n), var.memory_bytes(n), var.selection_flops(n), var.read_budget(n, 3),
                         var.memory_bytes(n, 3)])
    rec["accounting"] = np.array(acct, dtype=np.float64)
    np.savez_compressed(out / "csa2_variant.npz", **rec)


def make_nsa_variant(out):
    import torch
    from linattn.core import AttnConfig, block_reduce, repeat_kv
    from linattn.harness import structured_inputs
    from linattn.registry import build

    q, k, v = structured_inputs(1, 4, 192, 32, kv_heads=2, seed=9)
    q, k, v = q.float(), k.float(), v.float()
    cfg = AttnConfig(n_heads=4, n_kv_heads=2, head_dim=32, block_size=16, window_size=24, topk_blocks=3,
                     compress_ratio=8, seed=5)
    rec = {"fn": "NSAAttention", "q": _np(q), "k": _np(k), "v": _np(v)}
    with torch.no_grad():
        var = build("nsa", cfg)
        rec["gates_init"] = _np(var.gates.detach())
        rec["o_cmp"] = _np(var.branch_compression(q, k, v, 0))
        rec["o_slc"] = _np(var.branch_selection(q, k, v, 0))
        rec["o_win"] = _np(var.branch_window(q, k, v, 0))
        rec["sel_mask"] = _np(var.selection_mask(q, k, 0))
        kr = block_reduce(repeat_kv(k, 2), 16, -2)
        rec["block_scores"] = _np(torch.matmul(q, kr.transpose(-1, -2)) / (32 ** 0.5))
        for chunk in (64, 192):
            v2 = build("nsa", cfg)
            o, _ = v2.forward(q, k, v, chunk=chunk)
            rec[f"out{chunk}"] = _np(o)
            for key, val in v2.stats().items():
                rec[f"stats{chunk}_{key}"] = float(val)
        v3 = build("nsa", cfg)
        _, st = v3.forward(q[:, :, :191], k[:, :, :191], v[:, :, :191], chunk=191)
        od, _ = v3.forward(q[:, :, 191:], k[:, :, 191:], v[:, :, 191:], state=st)
        rec["out_decode"] = _np(od)
    # with one selected block every row's selection is defined (the own block is always
    # allowed, so the reference's top-k never reaches a later block): the full forward
    # and the learned gates (fit, then one forward in the learned mode)
    cfg1 = cfg.with_(topk_blocks=1)
    with torch.no_grad():
        v5 = build("nsa", cfg1)
        o, _ = v5.forward(q, k, v, chunk=192)
        rec["out192_k1"] = _np(o)
        rec["stats192_k1_selected_blocks_per_query"] = float(v5.stats()["selected_blocks_per_query"])
    v4 = build("nsa", cfg1)
    rec["fit_loss"] = float(v4.fit_gates(q, k, v, steps=25, lr=0.05))
    rec["gates_fit"] = _np(v4.gates.detach())
    with torch.no_grad():
        o, _ = v4.forward(q, k, v, chunk=192)
    rec["out_learned"] = _np(o)
    acct = []
    for extras in ({}, {"compress_ratio": 4, "selected_blocks": 6}):
        var = build("nsa", AttnConfig(n_heads=8, n_kv_heads=2, head_dim=64, extras=dict(extras)))
        for n in (5, 100, 4096):
            acct.append([var.read_budget(n), var.memory_bytes(n), var.flops(n), var.read_budget(n, 3),
                         var.memory_bytes(n, 3), var.flops(n, 3)])
    rec["accounting"] = np.array(acct, dtype=np.float64)
    np.savez_compressed(out / "nsa_variant.npz", **rec)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LINATTN_REF"),
                    help="root of the reference checkout (default: $LINATTN_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("the reference checkout is required: pass --ref or set LINATTN_REF")
    _import_reference(Path(args.ref))
    for fn in (make_page_bounds, make_page_select, make_topk_ties, make_quest_variant, make_block_sparse,
               make_indexer, make_dense, make_block_selectors, make_quant, make_paged_decode, make_dsa_variant,
               make_csa2_variant, make_nsa_variant):
        fn(HERE)
        print("wrote", fn.__name__)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
