#!/usr/bin/env python
"""Benchmark of the sparse-attention hot path on B200.

Workload ("quest_decode_c2"): paged Quest decode, one new token for each of B=16
sequences per GPU, H_q=32, H_kv=8, D=128, T=65536 per sequence in pages of 64
(1024 pages), bf16 KV with 1% needle pages along each kv group's query direction,
pages scattered by a seeded random permutation over a pool of 16x1024 pages; budget
32 pages + sink page 0 + the last page per query head (top-34 with both forced),
GQA union per kv head.  A step = page scoring + top-k/union + sparse attention
(split-KV + merge) for all 16 sequences; inputs resident in HBM, L2 flushed (a
256 MiB write, then a read of it, so no dirty line is left to write back) before
every step, outside the timed events.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
prints one JSON line.  For N > 1 (torchrun) every rank runs its own 16 sequences
(weak scaling, no data-path collective) and the step time is the max over ranks.
``--impl reference`` times the reference's CPU path on the host cores (rank 0 only).
At N = 1 the line also carries ``secondary``: config 4 (block selection + tcgen05
block-sparse causal prefill, B=2, T=131072; its TFLOP/s is ``prefill_tflops``) and
config 3 (lightning indexer + causal top-2048 + token attention, T=32768), each timed
with CUDA events over a few steps with the L2 flushed before each.

``--workload c3`` / ``--workload c4`` print config 3 / config 4 alone (one GPU;
``--seq-len`` shortens T for profiling captures).  ``--workload c5`` runs config 5 instead: B=64 sequences of 1,048,576 tokens (fp8 KV)
split across the N ranks (strong scaling), with NCCL all-gathers of the selection
candidates and of the partial (o, lse).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "sparse decode tok/s + HBM GB/s @64K ctx; prefill TFLOP/s @128K; % roofline"
C2 = dict(B=16, Hq=32, Hkv=8, D=128, T=65536, P=64, topk=34, sink_pages=1, needle_frac=0.01)
C3 = dict(B=1, T=32768, Hq=32, Hkv=8, D=128, HI=4, DI=64, topk=2048, scale_group=64)
C4 = dict(B=2, T=131072, Hq=32, Hkv=8, D=128, block=64, sink_blocks=1, window_blocks=16, topk=16, rank=8, amp=0.5)
C5 = dict(B=64, Hq=64, Hkv=8, D=128, T=1 << 20, P=64, topk=64, needle_frac=0.005)
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = ("flushed before every step, outside the timed events: a 256 MiB write, then a read of the same "
           "256 MiB so that the flush's dirty lines are written back before the step, not inside it")


def l2_flush(buf: torch.Tensor) -> None:
    """Write a buffer twice the L2 size, then read it back: L2 then holds only clean lines of
    the flush buffer (none of the step's data, and no write-back left for the step)."""
    buf.zero_()
    buf.view(torch.int64).amax()


# ---------------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------------
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


PROFILE_SOURCES = {  # the kernel source each traffic capture in profiles/ ran
    "sparse_attention_c2.md": "linattn_b200/csrc/sparse_attention_mma.cuh",
    "sparse_attention_c5.md": "linattn_b200/csrc/sparse_attention_mma.cuh",
    "quest_select_c5.md": "linattn_b200/csrc/quest_decode_select.cu",
}


def profile_traffic(name: str):
    """(DRAM bytes per launch, provenance) of a dominant kernel from the committed ncu
    summary ``profiles/<name>``: an ncu capture cannot run inside the timed bench, so the
    figure is the capture's, and ``source_match`` says whether the kernel source it ran
    (its sha256 is recorded in the summary) is the one in this tree."""
    import hashlib

    p = ROOT / "profiles" / name
    if not p.exists():
        return None, None
    value, captured = None, None
    for line in p.read_text().splitlines():
        line = line.strip()
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                value = float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                value = None
        elif line.startswith("kernel_source_sha256:"):
            captured = line.split(":", 1)[1].strip().split()[0]
    src = ROOT / PROFILE_SOURCES.get(name, "")
    current = hashlib.sha256(src.read_bytes()).hexdigest()[:16] if src.is_file() else None
    info = {"from": f"profiles/{name} (ncu capture)", "captured_source_sha256": captured,
            "current_source_sha256": current, "source_match": captured is not None and captured == current}
    return value, info


class ClockSampler:
    """SM clock and clock-event (throttle) reasons polled through NVML every ~2 ms
    while the timed region runs (the region can be far shorter than nvidia-smi's
    200 ms sampling period)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu, self.period = gpu_index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = None
        self._thread = None
        self.error = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as exc:  # noqa: BLE001
            self.error = f"nvml unavailable: {exc}"
            return self
        self._stop = threading.Event()

        def poll():
            while not self._stop.is_set():
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    bits = get_reasons(h)
                    for bit, name in self.REASONS.items():
                        if bits & bit:
                            self.reasons.add(name)
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(self.period)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if self.error:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": [self.error]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(self.reasons)}


# ---------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------
def build_c2(device, seed: int, n_q: int, batch: int = C2["B"]):
    """The config-2 cache on `device` plus `n_q` step queries (bf16)."""
    from linattn_b200 import PagedKVCache

    c = C2
    b, hq, hkv, d, t, p = batch, c["Hq"], c["Hkv"], c["D"], c["T"], c["P"]
    n_pages = t // p
    n_phys = b * n_pages
    gen = torch.Generator(device=device).manual_seed(seed)
    cache = PagedKVCache(b, hkv, d, p, n_pages, num_phys_pages=n_phys, dtype=torch.bfloat16, device=device)
    for s in range(0, n_phys, 1024):
        cache.k_pool[s:s + 1024].normal_(generator=gen)
        cache.v_pool[s:s + 1024].normal_(generator=gen)
    table = torch.randperm(n_phys, generator=gen, device=device).view(b, n_pages).to(torch.int32)
    q0 = torch.randn(b, hq, d, generator=gen, device=device)
    group = hq // hkv
    u = torch.nn.functional.normalize(q0.view(b, hkv, group, d).sum(2), dim=-1)  # (B, Hkv, D)
    n_needle = max(1, int(round(c["needle_frac"] * n_pages)))
    for bi in range(b):
        pages = torch.randperm(n_pages, generator=gen, device=device)[:n_needle]
        phys = table[bi, pages].long()
        add = (0.3 * math.sqrt(d)) * u[bi].view(1, hkv, 1, d)
        cache.k_pool[phys] = (cache.k_pool[phys].float() + add).to(torch.bfloat16)
    cache.set_page_table(table, [t] * b)
    cache.refresh_meta()
    qs = (q0.unsqueeze(0) + 0.25 * torch.randn(n_q, b, hq, d, generator=gen, device=device))
    qs = qs.view(n_q, b, hq, 1, d).to(torch.bfloat16)
    return cache, qs


def build_c5(device, rank: int, world: int, n_q: int, batch: int = C5["B"], t: int = C5["T"]):
    """This rank's shard of the config-5 cache (pages [lo, hi) of every sequence, fp8
    e4m3 with per-(page, kv head) scales, seeded N(0,1) values before quantisation,
    0.5% needle pages at global positions shared by all ranks, a random page table over
    the shard's pool) plus `n_q` step queries (identical on every rank)."""
    from linattn_b200 import PagedKVCache
    from linattn_b200.sharded import shard_page_ranges

    c = C5
    b, hq, hkv, d, p = batch, c["Hq"], c["Hkv"], c["D"], c["P"]
    n_glob = t // p
    lo, hi = shard_page_ranges(n_glob, world, rank)
    n_loc = hi - lo
    n_phys = b * n_loc
    cache = PagedKVCache(b, hkv, d, p, n_loc, num_phys_pages=n_phys, dtype=torch.float8_e4m3fn, device=device)
    gen = torch.Generator(device=device).manual_seed(5000 + rank)

    def quantise(x, pool, sc, at):
        amax = x.abs().amax(dim=(2, 3)).clamp_min(1e-8)
        scale = amax / torch.full_like(amax, 448.0)
        pool[at] = (x / scale[:, :, None, None]).to(torch.float8_e4m3fn).view(torch.uint8)
        sc[at] = scale

    chunk = 1024
    for s0 in range(0, n_phys, chunk):
        s1 = min(n_phys, s0 + chunk)
        for pool, sc in ((cache.k_pool, cache.k_scale), (cache.v_pool, cache.v_scale)):
            quantise(torch.randn(s1 - s0, hkv, p, d, generator=gen, device=device), pool, sc, slice(s0, s1))
    table = torch.randperm(n_phys, generator=gen, device=device).view(b, n_loc).to(torch.int32)
    gq = torch.Generator(device=device).manual_seed(4242)  # same stream on every rank
    q0 = torch.randn(b, hq, d, generator=gq, device=device)
    u = torch.nn.functional.normalize(q0.view(b, hkv, hq // hkv, d).sum(2), dim=-1)
    n_needle = max(1, int(round(c["needle_frac"] * n_glob)))
    for bi in range(b):
        pages = torch.randperm(n_glob, generator=gq, device=device)[:n_needle]
        mine = pages[(pages >= lo) & (pages < hi)] - lo
        if mine.numel() == 0:
            continue
        phys = table[bi, mine].long()
        x = cache.k_pool[phys].view(torch.float8_e4m3fn).float() * cache.k_scale[phys][:, :, None, None]
        quantise(x + (0.3 * math.sqrt(d)) * u[bi].view(1, hkv, 1, d), cache.k_pool, cache.k_scale, phys)
    cache.set_page_table(table, [n_loc * p] * b)
    cache.refresh_meta()
    qs = (q0.unsqueeze(0) + 0.25 * torch.randn(n_q, b, hq, d, generator=gq, device=device))
    return cache, qs.view(n_q, b, hq, 1, d).to(torch.bfloat16), (lo, hi)


def build_c4(device, seed: int, t: int = C4["T"]):
    """Config-4 inputs: Q/K N(0,1) plus a shared rank-8 component of amplitude 0.5, V N(0,1), bf16."""
    c = C4
    b, hq, hkv, d = c["B"], c["Hq"], c["Hkv"], c["D"]
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.randn(c["rank"], d, generator=g, device=device)

    def low_rank(x, h):
        # + amp * coef @ u, one rank-1 term at a time (elementwise: the input builder runs
        # no library GEMM, so launch lists of the workload hold this library's kernels)
        coef = torch.randn(b, h, t, c["rank"], generator=g, device=device)
        for r in range(c["rank"]):
            x.addcmul_(coef[..., r:r + 1], u[r], value=c["amp"])
        return x.to(torch.bfloat16)
    q = low_rank(torch.randn(b, hq, t, d, generator=g, device=device), hq)
    k = low_rank(torch.randn(b, hkv, t, d, generator=g, device=device), hkv)
    v = torch.randn(b, hkv, t, d, generator=g, device=device).to(torch.bfloat16)
    return q, k, v


def build_c3(device, seed: int, t: int = C3["T"]):
    """Config-3 inputs: bf16 Q/K/V N(0,1), indexer q/k N(0,1) with fp8 keys (per-64-token
    scales), indexer weights N(0, 1/64)."""
    from linattn_b200 import quantize_keys_fp8

    c = C3
    g = torch.Generator(device=device).manual_seed(seed)
    b = c["B"]
    q = torch.randn(b, c["Hq"], t, c["D"], generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(b, c["Hkv"], t, c["D"], generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(b, c["Hkv"], t, c["D"], generator=g, device=device).to(torch.bfloat16)
    q_idx = torch.randn(b, t, c["HI"], c["DI"], generator=g, device=device).to(torch.bfloat16)
    k_idx = torch.randn(b, t, c["HI"], c["DI"], generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(b, t, c["HI"], generator=g, device=device) / 8).to(torch.bfloat16)
    codes, scales = quantize_keys_fp8(k_idx, c["scale_group"])
    return q, k, v, q_idx, codes, scales, w


def _time_events(fn_parts, steps: int, warmup: int, flush, stream):
    """Runs the phases of one step (callables) `warmup` + `steps` times with an L2 flush
    before every step; returns the mean ms of each phase over the timed steps."""
    for _ in range(warmup):
        l2_flush(flush)
        for f in fn_parts:
            f()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fn_parts) + 1)] for _ in range(steps)]
    for i in range(steps):
        l2_flush(flush)
        ev[i][0].record(stream)
        for j, f in enumerate(fn_parts):
            f()
            ev[i][j + 1].record(stream)
    torch.cuda.synchronize()
    return [statistics.mean(ev[i][j].elapsed_time(ev[i][j + 1]) for i in range(steps)) for j in range(len(fn_parts))]


def secondary_c4(device, steps: int, warmup: int, flush, stream, t: int = C4["T"], parity: bool = True):
    """Config 4 on this GPU: block selection + block-sparse causal prefill (tcgen05)."""
    from linattn_b200.blocks import block_select, block_sparse_prefill

    c = C4
    q, k, v = build_c4(device, 44, t)
    res = {}

    def sel():
        res["ids"], res["cnt"] = block_select(q, k, c["block"], c["topk"], sink_blocks=c["sink_blocks"],
                                              window_blocks=c["window_blocks"])
    sel()
    out = torch.empty_like(q)

    def att():
        block_sparse_prefill(q, k, v, res["ids"], counts=res["cnt"], rows_per_list=c["block"], out=out)
    ms_sel, ms_att = _time_events([sel, att], steps, warmup, flush, stream)
    par = None
    if parity:
        torch.cuda.synchronize(device)
        par = parity_block_prefill(q, k, v, res["ids"], res["cnt"], out, c["block"], c["topk"], c["sink_blocks"],
                                   c["window_blocks"])
    cnt = res["cnt"].long()
    bs, d = c["block"], c["D"]
    # allowed (query, key) pairs, causal-exact: full 64x64 blocks off the diagonal, a triangle on it
    pairs = (cnt - 1).sum().item() * bs * bs + c["B"] * c["Hq"] * (t // bs) * (bs * (bs + 1) // 2)
    flops = 4 * d * pairs
    _, peak, kind = measured_peaks()
    tfl = flops / (ms_att * 1e-3) / 1e12
    return {"workload": "block_sparse_prefill_c4", "B": c["B"], "T": t, "select_ms": round(ms_sel, 3),
            "prefill_ms": round(ms_att, 3), "prefill_tflops": round(tfl, 1), "frac_of_bf16_peak": round(tfl / peak, 4),
            "peak_kind": kind, "mean_blocks_per_query_block": round(cnt.float().mean().item(), 2),
            "algorithmic_flops": int(flops), "end_to_end_tflops": round(flops / ((ms_sel + ms_att) * 1e-3) / 1e12, 1),
            "launches_per_step": 6, **({"parity": par} if par is not None else {})}


def measure_read_gbs(device, mib: int, reps: int) -> float:
    """Read roof of a `mib` MiB buffer: `linattn_read_bandwidth` (a persistent grid of
    16-byte loads, eight in flight per thread) timed with CUDA events after a warm-up
    pass; a buffer that fits the 126 MB L2 gives the L2 read roof, a larger one HBM's."""
    from linattn_b200 import _lib as L

    n = mib << 20
    buf = torch.empty(n, dtype=torch.uint8, device=device).random_(0, 255)
    sink = torch.zeros(1024, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)

    def run(r):
        L.check(L.lib().linattn_read_bandwidth(buf.data_ptr(), n, r, sink.data_ptr(), sink.numel(),
                                               stream.cuda_stream))
    run(2)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run(reps)
    e1.record()
    torch.cuda.synchronize(device)
    return n * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9


def secondary_c3(device, steps: int, warmup: int, flush, stream, t: int = C3["T"], parity: bool = True):
    """Config 3 on this GPU: lightning indexer + causal top-2048 + token attention."""
    from linattn_b200 import indexer_topk
    from linattn_b200.dsa import token_sparse_attention

    c = C3
    q, k, v, q_idx, codes, scales, w = build_c3(device, 33, t)
    res = {}

    def sel():
        _, res["ids"] = indexer_topk(q_idx, codes, w, c["topk"], causal=True, k_scale=scales,
                                     scale_group=c["scale_group"], index_dtype=torch.int32, sorted=False)
    sel()
    out = torch.empty_like(q)

    def att():
        token_sparse_attention(q, k, v, res["ids"].unsqueeze(1), causal=True, out=out)
    ms_sel, ms_att = _time_events([sel, att], steps, warmup, flush, stream)
    par = None
    if parity and t >= 4096:
        torch.cuda.synchronize(device)
        par = parity_dsa(q, k, v, q_idx, codes, scales, w, res["ids"], out, c["topk"], c["scale_group"])
    kk, d = c["topk"], c["D"]
    vis = sum(min(i + 1, kk) for i in range(t))  # selected tokens per query, causal
    gather = vis * c["Hkv"] * d * 2 * 2
    l2 = measure_read_gbs(device, 48, 200)
    return {"workload": "dsa_indexer_attention_c3", "T": t, "select_ms": round(ms_sel, 3),
            "attention_ms": round(ms_att, 3), "total_ms": round(ms_sel + ms_att, 3),
            "attention_gathered_gbs": round(gather / (ms_att * 1e-3) / 1e9, 1),
            "l2_read_gbs": round(l2, 1),
            "attention_gathered_frac_of_l2": round(gather / (ms_att * 1e-3) / 1e9 / l2, 4),
            "peak_kind": "measured in this run: linattn_read_bandwidth over a 48 MiB L2-resident buffer (the gathered "
                         "K/V rows of one batch, 134 MB, sit in the 126 MB L2 almost whole: 99.8% hit rate)",
            "attention_tflops": round(4 * c["Hq"] * d * vis / (ms_att * 1e-3) / 1e12, 1),
            "launches_per_step": 2 * -(-t // max(1, min(t, (1 << 29) // (t * 4)))) + 1,
            **({"parity": par} if par is not None else {})}


def run_prefill_workload(args):
    """Config 3 or 4 alone on one GPU (``--workload c3|c4``; ``--seq-len`` shortens T for
    profiling captures): one JSON line with the prefill's own metric and roofline."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    hbm, peak, kind = measured_peaks()
    base = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1); config-4 Q/K with a shared "
            "rank-8 component)", "gpu_launches": None}
    with ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])) as clocks:
        if args.workload == "c4":
            t = args.seq_len or C4["T"]
            r = secondary_c4(device, args.steps, args.warmup, flush, stream, t, parity=not args.no_parity)
            par = r.pop("parity", None)
            line = dict(base, metric="block-sparse causal prefill TFLOP/s", value=r["prefill_tflops"], unit="TFLOP/s",
                        ms_per_step=r["prefill_ms"],
                        config={"workload": "block_sparse_prefill_c4" if t == C4["T"] else f"block_sparse_prefill_c4_t{t}",
                                "l2": L2_NOTE, **C4,
                                "T": t},
                        roofline={"bound": "tensor", "kernel": "prefill_umma_kernel", "achieved": r["prefill_tflops"],
                                  "peak": peak, "unit": "TFLOP/s", "frac": r["frac_of_bf16_peak"], "peak_kind": kind,
                                  "traffic": None, "algorithmic_flops_per_launch": r["algorithmic_flops"]},
                        detail=r)
            line["gpu_launches"] = r["launches_per_step"] * args.steps
        else:
            t = args.seq_len or C3["T"]
            r = secondary_c3(device, args.steps, args.warmup, flush, stream, t, parity=not args.no_parity)
            par = r.pop("parity", None)
            line = dict(base, metric="DSA prefill tok/s", value=round(t / (r["total_ms"] * 1e-3), 1), unit="tok/s",
                        ms_per_step=r["total_ms"],
                        config={"workload": "dsa_indexer_attention_c3" if t == C3["T"] else f"dsa_c3_t{t}",
                                "l2": L2_NOTE, **C3,
                                "T": t},
                        roofline={"bound": "l2", "kernel": "token_attention_kernel (gathered rows; L2 hits)",
                                  "achieved": r["attention_gathered_gbs"], "peak": r["l2_read_gbs"], "unit": "GB/s",
                                  "frac": r["attention_gathered_frac_of_l2"], "peak_kind": r["peak_kind"],
                                  "traffic": None},
                        detail=r)
            line["gpu_launches"] = r["launches_per_step"] * args.steps
    line["clocks"] = clocks.summary()
    if par is not None:
        line["parity"] = {line["config"]["workload"]: par}
    return line


CV = dict(B=1, T=16384, Hq=32, Hkv=8, D=128, csa2_ratio=16, csa2_topk_groups=64, csa2_window=256, csa2_bits=4,
          nsa_block=64, nsa_selected=16, nsa_window=512, nsa_compress=16)


def run_variants_workload(args):
    """The CSA2 and NSA plugins' prefill forward on one GPU (``--workload variants``):
    per-phase CUDA-event times, the pool + codec kernel's HBM bandwidth, the CSA2
    attention's gathered bandwidth and the NSA selection branch's TFLOP/s.  Not part of
    the default run."""
    from linattn_b200.core import AttnConfig
    from linattn_b200.registry import build

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    hbm, peak, kind = measured_peaks()
    c = CV
    b, hq, hkv, t, d = c["B"], c["Hq"], c["Hkv"], args.seq_len or c["T"], c["D"]
    g = torch.Generator(device=device).manual_seed(77)
    q, k, v = (torch.randn(b, h, t, d, device=device, generator=g, dtype=torch.float32).to(torch.bfloat16)
               for h in (hq, hkv, hkv))
    with ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])) as clocks:
        # ---- CSA2
        csa = build("cuda_csa2", AttnConfig(n_heads=hq, n_kv_heads=hkv, head_dim=d, seed=1,
                                            extras={"compress_ratio": c["csa2_ratio"], "bits": c["csa2_bits"],
                                                    "topk_groups": c["csa2_topk_groups"], "window": c["csa2_window"]}))
        st = {}

        def pool():
            st["kv"] = csa.compressed_kv(k, v)

        def select():
            st["ids"] = csa.select_groups(q, st["kv"][0], t, 0)

        def attend():
            st["o"] = csa.attend_kv(q, k, v, compressed=st["kv"])
        pool()
        select()
        ms_pool, ms_sel, ms_att = _time_events([pool, select, attend], args.steps, args.warmup, flush, stream)
        reads = csa.stats()["reads_per_query"]
        n_groups = st["kv"][0].shape[2]
        pool_bytes = 2 * (b * hkv * t * d * 2 + b * hkv * n_groups * d * 2)
        gathered = reads * b * hkv * t * 2 * d * 2  # K and V rows per (query, kv head)
        ms_attention = max(ms_att - ms_sel, 1e-9)
        csa2 = {"pool_quant_ms": round(ms_pool, 4), "select_ms": round(ms_sel, 4),
                "attend_ms (selection + attention)": round(ms_att, 4), "total_ms": round(ms_pool + ms_att, 4),
                "tok_per_s": round(b * t / ((ms_pool + ms_att) * 1e-3), 1),
                "pool_quant_gbs": round(pool_bytes / (ms_pool * 1e-3) / 1e9, 1),
                "pool_quant_frac_of_hbm": round(pool_bytes / (ms_pool * 1e-3) / 1e9 / hbm, 4),
                "reads_per_query": round(reads, 2), "groups_per_query": round(csa.stats()["groups_per_query"], 2),
                "attention_gathered_gbs": round(gathered / (ms_attention * 1e-3) / 1e9, 1)}
        # ---- NSA
        nsa = build("cuda_nsa", AttnConfig(n_heads=hq, n_kv_heads=hkv, head_dim=d, seed=1, block_size=c["nsa_block"],
                                           window_size=c["nsa_window"], topk_blocks=c["nsa_selected"],
                                           compress_ratio=c["nsa_compress"]))
        outs = torch.empty(3, *q.shape, dtype=torch.float32, device=device)
        ns = {}

        def cmp_():
            nsa.branch_compression(q, k, v, 0, out=outs[0])

        def sel_lists():
            ns["lists"] = nsa.selection_lists(q, k, 0)

        def slc():
            nsa.branch_selection(q, k, v, 0, out=outs[1])

        def win():
            nsa.branch_window(q, k, v, 0, out=outs[2])

        def full():
            nsa.attend(q, {"k": k, "v": v}, 0)
        sel_lists()
        ms_c, ms_l, ms_s, ms_w, ms_f = _time_events([cmp_, sel_lists, slc, win, full], args.steps, args.warmup, flush,
                                                    stream)
        counts = ns["lists"][1].long()
        pairs = counts.sum().item() * c["nsa_block"]  # whole blocks are read
        slc_tfl = 4 * d * pairs / (max(ms_s - ms_l, 1e-9) * 1e-3) / 1e12
        nsa_r = {"compression_branch_ms": round(ms_c, 4), "selection_lists_ms": round(ms_l, 4),
                 "selection_branch_ms (lists + attention)": round(ms_s, 4), "window_branch_ms": round(ms_w, 4),
                 "attend_ms": round(ms_f, 4), "tok_per_s": round(b * t / (ms_f * 1e-3), 1),
                 "selected_blocks_per_query": round(counts.float().mean().item(), 2),
                 "selection_attention_tflops": round(slc_tfl, 1), "selection_attention_frac_of_bf16_peak":
                     round(slc_tfl / peak, 4)}
    line = {"metric": "CSA2 / NSA prefill tok/s", "value": csa2["tok_per_s"], "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": csa2["total_ms"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "csa2_nsa_prefill", "l2": L2_NOTE, **c, "T": t},
            "roofline": {"bound": "hbm", "kernel": "csa2_pool_quant_vec_kernel", "achieved": csa2["pool_quant_gbs"],
                         "peak": hbm, "unit": "GB/s", "frac": csa2["pool_quant_frac_of_hbm"], "peak_kind": kind,
                         "traffic": None},
            "detail": {"csa2": csa2, "nsa": nsa_r}, "gpu_launches": None, "clocks": clocks.summary()}
    return line


# ---------------------------------------------------------------------------------
# full-size parity: checker legs on samples of the benchmarked workloads, outside the
# timed regions (the CPU oracle is the checker here, never the thing measured)
# ---------------------------------------------------------------------------------
TOL_16, TOL_FP8 = 2e-3, 1e-2  # north_star: bf16 / f16 inputs, fp8 KV (against the dequantised KV)


def _out_errors(got_out: np.ndarray, ref: np.ndarray, tol: float, out_dtype, got32=None) -> dict:
    """Errors against the float64 oracle: the fp32-domain result (when given) against the
    bare tolerance, and the result in its output dtype against the tolerance plus half an
    ulp of that dtype at |ref| (the one rounding to bf16 / f16 alone reaches that)."""
    half = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}.get(out_dtype, 0.0)
    e = np.abs(got_out - ref)
    res = {"tol": tol, "max_abs_out": float(e.max()), "ok_out": bool(np.all(e <= tol + half * np.abs(ref)))}
    if got32 is not None:
        e32 = float(np.abs(got32 - ref).max())
        res.update({"max_abs_fp32": e32, "ok_fp32": e32 <= tol})
    return res


def _union_attention_oracle(cache, qn, lens, uids, cnt, scale):
    """Float64 oracle attention over each (sequence, kv head)'s union pages, one
    (sequence, kv head) at a time with only its pages copied to the host (fp8 codes
    decoded and scaled by the oracle), so the whole pool never leaves the device."""
    import oracle

    n, hq, d = qn.shape
    hkv, p = cache.n_kv_heads, cache.page_size
    group = hq // hkv
    ref = np.zeros((n, hq, d))
    for bi in range(n):
        for kh in range(hkv):
            pages = uids[bi, kh, : cnt[bi, kh]].astype(np.int64)
            phys = cache.page_table[bi].long()[torch.from_numpy(pages).to(cache.device)]
            kk = cache.k_pool[phys, kh]
            vv = cache.v_pool[phys, kh]
            if cache.fp8:
                kk, vv = kk.view(torch.float8_e4m3fn), vv.view(torch.float8_e4m3fn)
            kp = kk.float().cpu().numpy()[:, None]                  # (n_u, 1, P, D)
            vp = vv.float().cpu().numpy()[:, None]
            ks = cache.k_scale[phys, kh].cpu().numpy()[:, None] if cache.fp8 else None
            vs = cache.v_scale[phys, kh].cpu().numpy()[:, None] if cache.fp8 else None
            table = np.zeros((1, int(pages.max()) + 1 if pages.size else 1), dtype=np.int64)
            table[0, pages] = np.arange(pages.size)
            ref[bi, kh * group:(kh + 1) * group] = oracle.paged_sparse_decode(
                qn[bi:bi + 1, kh * group:(kh + 1) * group], kp, vp, table, lens[bi:bi + 1],
                pages[None, None], np.array([[pages.size]]), page_size=p, scale=scale, k_scale=ks, v_scale=vs)[0]
    return ref


def parity_quest_decode(cache, q, topk: int, sink_pages: int, *, n_splits: int, force_last: bool = True,
                        timed_out=None, n_check: int = 2, tol: float = TOL_16):
    """The decode step at full size on sequences [0, n_check): the page bounds exactly
    against the oracle (16-bit pools); the kernel's fp32 page scores against the float64
    oracle on the stored bounds; the selected pages bit-exact against the oracle's
    lowest-index top-k on the kernel's own scores; the GQA union; the attention over
    the union against the float64 oracle (fp32 output against the bare tolerance, the
    q-dtype output with half an ulp); and ``timed_out`` (the timed decoder's output for
    the same q) equal to this checking decoder's."""
    import oracle
    from linattn_b200 import QuestDecoder
    from linattn_b200.block_sparse import sparse_attention

    hq = q.shape[1]
    hkv, p, d = cache.n_kv_heads, cache.page_size, cache.head_dim
    group = hq // hkv
    chk = QuestDecoder(cache, hq, topk, sink_pages=sink_pages, q_dtype=q.dtype, keep_scores=True,
                       force_last=force_last, n_splits=n_splits)
    out_chk = chk.step(q).clone()
    o32 = sparse_attention(q, cache.kv_desc(), chk._lists, scale=chk.scale,
                           out=torch.empty(q.shape, dtype=torch.float32, device=q.device), n_splits=chk.n_splits)
    torch.cuda.synchronize(q.device)
    lens = cache.seq_lens[:n_check].cpu().numpy().astype(np.int64)
    n_b = (lens + p - 1) // p
    scores = chk.scores[:n_check].cpu().numpy().astype(np.float64)
    ids = chk.ids[:n_check].cpu().numpy().astype(np.int64)
    cnt = chk.union_count[:n_check, :, 0].cpu().numpy()
    uids = chk.union_ids[:n_check, :, 0].cpu().numpy()
    sets_equal, union_equal, bounds_exact, score_rel = True, True, True, 0.0
    mins = cache.meta_min[:n_check].float().cpu().numpy()  # (n, H_kv, pages, D), logical order
    maxs = cache.meta_max[:n_check].float().cpu().numpy()
    qn = q[:n_check].float().cpu().numpy()
    for bi in range(n_check):
        kb = max(1, min(topk, int(n_b[bi])))
        want = oracle.topk_lowest_index(scores[bi, :, :, : n_b[bi]], kb)
        sets_equal &= bool(np.array_equal(ids[bi, :, :, :kb], want))
        union = oracle.gqa_union(ids[bi:bi + 1, :, :, :kb], int(n_b[bi]), group)[0, :, 0]
        for kh in range(hkv):
            union_equal &= bool(np.array_equal(uids[bi, kh, : cnt[bi, kh]], np.nonzero(union[kh])[0]))
        for kh in range(hkv):  # one kv head at a time (float64 temporaries stay small)
            hs = slice(kh * group, (kh + 1) * group)
            ref_s = oracle.page_scores(qn[bi:bi + 1, hs], mins[bi:bi + 1, kh:kh + 1, : n_b[bi]],
                                       maxs[bi:bi + 1, kh:kh + 1, : n_b[bi]])[0]
            got_s = scores[bi, hs, :, : n_b[bi]]
            fin = np.isfinite(got_s)
            score_rel = max(score_rel, float((np.abs(got_s - ref_s)[fin] / (np.abs(ref_s[fin]) + 1.0)).max()))
        if not cache.fp8:
            # page bounds: every page of the sequence, exact (min / max of 16-bit values)
            tab = cache.page_table[bi, : n_b[bi]].long()
            kk = cache.k_pool[tab].float().cpu().numpy()  # (pages, H_kv, P, D)
            bn, bx = oracle.page_bounds(kk.transpose(1, 0, 2, 3).reshape(1, hkv, -1, d)[:, :, : lens[bi]], p)
            bounds_exact &= bool(np.array_equal(bn[0], mins[bi, :, : n_b[bi]]) and
                                 np.array_equal(bx[0], maxs[bi, :, : n_b[bi]]))
    ref = _union_attention_oracle(cache, qn[:, :, 0], lens, uids, cnt, chk.scale)
    res = {"sequences_checked": n_check, "sets_equal": sets_equal, "union_equal": union_equal,
           "bounds_exact": bounds_exact if not cache.fp8 else None, "score_max_rel_err": score_rel,
           "timed_output_equal": None if timed_out is None else bool(torch.equal(out_chk, timed_out))}
    res.update(_out_errors(out_chk[:n_check, :, 0].float().cpu().numpy(), ref, tol, q.dtype,
                           o32[:n_check, :, 0].cpu().numpy()))
    if timed_out is not None:
        # the timed decoder's own output for the same q, against the same oracle
        res["timed_ok_out"] = _out_errors(timed_out[:n_check, :, 0].float().cpu().numpy(), ref, tol,
                                          timed_out.dtype)["ok_out"]
    res["ok"] = bool(sets_equal and union_equal and res["ok_out"] and res["ok_fp32"]
                     and res.get("timed_ok_out", True) and (cache.fp8 or bounds_exact))
    return res


def parity_block_prefill(q, k, v, ids, cnt, out, block: int, topk: int, sink_blocks: int, window_blocks: int,
                         n_qb_check: int = 8, tol: float = TOL_16):
    """Config 4 at full size on ``n_qb_check`` query blocks spread over T (the first and
    the last included), every (b, head): the block lists bit-exact against the oracle's
    rule (sink + window + lowest-index top-k of the causal candidates) applied to the
    kernel's own fp32 pooled scores (recorded for those rows by the same kernel); the
    same rule on float64 pooled scores, where a row may differ only at a near tie
    (k-th and (k+1)-th candidate within 1e-5 relative); and the prefill output against
    float64 attention over the kernel's own lists with the causal rule."""
    from linattn_b200.blocks import block_mean, block_score_topk

    b, hq, t, d = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    n_qb = t // block
    qbs = sorted(set(np.linspace(0, n_qb - 1, n_qb_check).round().astype(int).tolist()))
    ids_h = ids.cpu().numpy()
    cnt_h = cnt.cpu().numpy()
    qp, kp = block_mean(q, block), block_mean(k, block)
    kmean = kp.double().cpu().numpy()          # the fp32 means, as float64
    exact_mismatch, f64_mismatch, near_ties, rows = 0, 0, 0, 0
    err_max, ok_out = 0.0, True
    half = 2.0 ** -8
    for qb in qbs:
        own_sc = torch.full((b, hq, 1, n_qb), float("-inf"), device=q.device)
        block_score_topk(qp[:, :, qb:qb + 1], kp, topk, scale=1.0 / math.sqrt(d), first_pos=qb - window_blocks,
                         key_block=1, skip=sink_blocks, merge_pos=qb, sink=sink_blocks, window=window_blocks,
                         scores_out=own_sc)
        own_sc = own_sc[:, :, 0].double().cpu().numpy()                            # (B, Hq, n_qb)
        qmean = qp[:, :, qb].double().cpu().numpy()                                # (B, Hq, D)
        sc64 = np.einsum("bhgd,bhkd->bhgk", qmean.reshape(b, hkv, group, d), kmean).reshape(b, hq, n_qb)
        sc64 /= math.sqrt(d)
        q_blk = q[:, :, qb * block:(qb + 1) * block].double().cpu().numpy()      # (B, Hq, 64, D)
        kbi = np.arange(n_qb)
        cand_ok = (kbi >= sink_blocks) & (kbi <= qb - window_blocks)
        forced = ((kbi < sink_blocks) | (kbi > qb - window_blocks)) & (kbi <= qb)
        for bi in range(b):
            for h in range(hq):
                got = np.sort(ids_h[bi, h, qb, : cnt_h[bi, h, qb]])
                rows += 1
                for scores, kind in ((own_sc[bi, h], "own"), (sc64[bi, h], "f64")):
                    cand = np.where(cand_ok, scores, -np.inf)
                    order = np.argsort(-cand, kind="stable")
                    kk = min(topk, int(cand_ok.sum()))
                    want = np.sort(np.concatenate([np.nonzero(forced)[0], order[:kk]]))
                    if np.array_equal(got, want):
                        continue
                    if kind == "own":
                        exact_mismatch += 1
                    else:
                        srt = cand[order]
                        if kk < srt.size and np.isfinite(srt[kk]) and abs(srt[kk - 1] - srt[kk]) <= 1e-5 * (
                                abs(srt[kk]) + 1e-6):
                            near_ties += 1
                        else:
                            f64_mismatch += 1
                kh = h // group
                tok = (got[:, None] * block + np.arange(block)[None, :]).reshape(-1)
                sel = torch.from_numpy(tok).to(k.device)
                kk_ = k[bi, kh, sel].double().cpu().numpy()
                vv_ = v[bi, kh, sel].double().cpu().numpy()
                pos = qb * block + np.arange(block)
                allow = tok[None, :] <= pos[:, None]
                sco = (q_blk[bi, h] @ kk_.T) / math.sqrt(d)
                sco = np.where(allow, sco, -np.inf)
                sco -= sco.max(-1, keepdims=True)
                pw = np.exp(sco)
                ref = (pw @ vv_) / pw.sum(-1, keepdims=True)
                got_o = out[bi, h, qb * block:(qb + 1) * block].float().cpu().numpy()
                e = np.abs(got_o - ref)
                err_max = max(err_max, float(e.max()))
                ok_out &= bool(np.all(e <= tol + half * np.abs(ref)))
    return {"query_blocks_checked": qbs, "rows_checked": rows, "sets_equal": exact_mismatch == 0,
            "sets_mismatch_own_scores": exact_mismatch, "sets_mismatch_float64": f64_mismatch,
            "near_tie_rows_float64": near_ties, "tol": tol, "max_abs_out": err_max, "ok_out": ok_out,
            "ok": bool(ok_out and exact_mismatch == 0)}


def parity_dsa(q, k, v, q_idx, codes, scales, w, ids, out, topk: int, scale_group: int, tol: float = TOL_16):
    """Config 3 at full size on 64 query rows in runs of 8 spread over T (t < 2048,
    across 2048 and t = T-1 included): the kernel's fp32 indexer scores for those rows
    against the float64 oracle on the dequantised fp8 keys; the selected tokens
    bit-exact against the oracle's lowest-index causal top-k on the kernel's own
    scores; the attention against float64 attention over the selected tokens."""
    import oracle
    from linattn_b200 import indexer_scores

    b, hq, t, d = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    # runs of 8 rows; at a shortened T (profiling captures) the runs past it are left out
    starts = sorted({r for r in (0, 1000, 2044, 4100, 9000, 16380, 24000) if r + 8 <= t} | {max(0, t - 8)})
    kdq = codes.view(torch.uint8).cpu().numpy()
    kdq = oracle.e4m3_decode(kdq).astype(np.float64)
    sc_h = scales.cpu().numpy()
    sets_equal, score_rel, err_max, ok_out, rows = True, 0.0, 0.0, True, 0
    ids_h = ids.cpu().numpy()
    for r0 in starts:
        r1 = r0 + 8
        s = indexer_scores(q_idx[:, r0:r1], codes, w[:, r0:r1], k_scale=scales, scale_group=scale_group,
                           causal=True, offset=r0)
        got_s = s.cpu().numpy().astype(np.float64)                                 # (B, 8, T)
        ref_s = oracle.indexer_scores(q_idx[:, r0:r1].float().cpu().numpy(), kdq, w[:, r0:r1].float().cpu().numpy(),
                                      k_scale=sc_h, group=scale_group)
        for i in range(r1 - r0):
            tq = r0 + i
            vis = tq + 1
            fin = got_s[0, i, :vis]
            score_rel = max(score_rel, float((np.abs(fin - ref_s[0, i, :vis]) / (np.abs(ref_s[0, i, :vis]) + 1.0)).max()))
            kk = min(topk, vis)
            want = np.sort(oracle.topk_lowest_index(fin, kk))
            got = np.sort(ids_h[0, tq][ids_h[0, tq] >= 0])
            sets_equal &= bool(np.array_equal(got, want))
            rows += 1
            sel = torch.from_numpy(got).to(k.device)
            qq = q[0, :, tq].double().cpu().numpy()                                # (Hq, D)
            for kh in range(hkv):
                kk_ = k[0, kh, sel].double().cpu().numpy()
                vv_ = v[0, kh, sel].double().cpu().numpy()
                sco = qq[kh * group:(kh + 1) * group] @ kk_.T / math.sqrt(d)
                sco -= sco.max(-1, keepdims=True)
                pw = np.exp(sco)
                ref = pw @ vv_ / pw.sum(-1, keepdims=True)
                got_o = out[0, kh * group:(kh + 1) * group, tq].float().cpu().numpy()
                e = np.abs(got_o - ref)
                err_max = max(err_max, float(e.max()))
                ok_out &= bool(np.all(e <= tol + 2.0 ** -8 * np.abs(ref)))
    return {"rows_checked": rows, "row_starts": starts, "sets_equal": sets_equal, "score_max_rel_err": score_rel,
            "tol": tol, "max_abs_out": err_max, "ok_out": ok_out, "ok": bool(sets_equal and ok_out)}


# ---------------------------------------------------------------------------------
# CPU baselines: the reference's own torch operators on the host cores
# ---------------------------------------------------------------------------------
REF_DIR = ROOT / "baseline" / "_ref"


def reference_ops():
    """The reference's CPU torch operators for the Quest decode path, imported from
    its unmodified install in ``baseline/_ref`` (never this library):
    ``page_bounds_torch`` / ``page_select_torch`` (``kernels/triton/quest_pages.py:38-78``)
    and ``block_sparse_attention_torch`` (``kernels/triton/block_sparse.py:40-75``)."""
    if not (REF_DIR / "linattn" / "__init__.py").exists():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from linattn.kernels.triton.block_sparse import block_sparse_attention_torch
    from linattn.kernels.triton.quest_pages import page_bounds_torch, page_select_torch

    return page_bounds_torch, page_select_torch, block_sparse_attention_torch


def reference_quest_step(ops, q, k, v, mins, maxs, page: int, topk: int, sink_pages: int, group: int):
    """One config-2 decode step through the reference's operators, fp32 on the CPU:
    the per-page bounds are repeated over each kv group's query heads (as
    ``QuestAttention.page_scores`` does with ``repeat_kv``, ``variants/selection.py:203-212``),
    ``page_select_torch`` takes the top-``topk`` pages with the query's own (last) page
    forced, the sink page is forced the same way (it replaces the lowest-ranked pick
    when it is not already chosen), the heads of a group read the union of their
    pages (``selection.py:232-235``), and ``block_sparse_attention_torch`` attends over
    the union (padding ids point past the end and are masked by the operator)."""
    _, page_select_torch, block_sparse_attention_torch = ops
    b, hq, _, d = q.shape
    hkv, t = k.shape[1], k.shape[2]
    n_pages = mins.shape[2]
    ids, _ = page_select_torch(q, mins.repeat_interleave(group, dim=1), maxs.repeat_interleave(group, dim=1), page,
                               topk, offset=t - 1)
    ids = ids[:, :, 0]                                                   # (B, Hq, topk), score order
    if sink_pages:
        assert sink_pages == 1
        ids[..., -1] = torch.where((ids == 0).any(-1), ids[..., -1], torch.zeros_like(ids[..., -1]))
    sel = torch.zeros(b, hq, n_pages, dtype=torch.bool).scatter_(-1, ids, True)
    union = sel.view(b, hkv, group, n_pages).any(2)                      # (B, Hkv, n_pages)
    n_max = int(union.sum(-1).max())
    order = torch.where(union, torch.arange(n_pages), torch.full((), n_pages)).sort(-1).values[..., :n_max]
    out = block_sparse_attention_torch(q, k, v, order, block_size=page)
    return out, union


def build_c2_host(seed: int, n_q: int, batch: int, threads: int):
    """The config-2 workload built on the host (numpy, no GPU): the same construction
    as ``build_c2`` (N(0,1) K/V rounded to bf16, 1% needle pages with
    0.3*sqrt(D)*(unit group q direction) added to their keys, queries around a base
    query) from host generators; contiguous ``(B, H_kv, T, D)`` fp32 tensors holding
    bf16 values, the reference's layout (it has no page table)."""
    c = C2
    b, hq, hkv, d, t, p = batch, c["Hq"], c["Hkv"], c["D"], c["T"], c["P"]
    group = hq // hkv
    n_pages = t // p

    def bf16_round(x):
        u = x.view(np.uint32)
        u += np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))
        u &= np.uint32(0xFFFF0000)
        return x

    seqs = np.random.SeedSequence(seed).spawn(2 * b * hkv + 1)
    kv = np.empty((2, b, hkv, t, d), dtype=np.float32)

    def fill(i):
        x = kv.reshape(2 * b * hkv, t, d)[i]
        np.random.default_rng(seqs[i]).standard_normal(out=x, dtype=np.float32)
        bf16_round(x)
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(fill, range(2 * b * hkv)))
    rng = np.random.default_rng(seqs[-1])
    q0 = rng.standard_normal((b, hq, d), dtype=np.float32)
    u = q0.reshape(b, hkv, group, d).sum(2)
    u /= np.linalg.norm(u, axis=-1, keepdims=True)
    n_needle = max(1, int(round(c["needle_frac"] * n_pages)))
    k = kv[0]
    for bi in range(b):
        for pg in rng.permutation(n_pages)[:n_needle]:
            blk = k[bi, :, pg * p:(pg + 1) * p]
            blk += (0.3 * math.sqrt(d)) * u[bi][:, None, :]
            bf16_round(blk)
    qs = q0[None] + 0.25 * rng.standard_normal((n_q, b, hq, d), dtype=np.float32)
    bf16_round(qs)
    return (torch.from_numpy(kv[0]), torch.from_numpy(kv[1]),
            torch.from_numpy(np.ascontiguousarray(qs)).view(n_q, b, hq, 1, d))


def cpu_reference_step_fn(cache, q, n_seq: int, threads: int):
    """Returns (fn, kind, description): fn() runs one CPU step over a sample of this
    run's own config-2 data (sequences [0, n_seq), host copies in the reference's
    contiguous fp32 layout).  With the reference installed (``baseline/_ref``) the step
    is ``reference_quest_step`` (kind "reference"); without it, the oracle's C
    restatement of the same step (kind "port")."""
    c = C2
    hq, hkv, d, p, t = c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    n_pages = t // p
    group = hq // hkv
    tab = cache.page_table[:n_seq].long().flatten()
    kp = cache.k_pool[tab].float().cpu()                       # (n_seq*n_pages, Hkv, P, D)
    vp = cache.v_pool[tab].float().cpu()
    k = kp.view(n_seq, n_pages, hkv, p, d).transpose(1, 2).reshape(n_seq, hkv, t, d).contiguous()
    v = vp.view(n_seq, n_pages, hkv, p, d).transpose(1, 2).reshape(n_seq, hkv, t, d).contiguous()
    qf = q[:n_seq].float().cpu().contiguous()
    ops = reference_ops()
    torch.set_num_threads(threads)
    if ops is not None:
        mins, maxs = ops[0](k, p)

        def reference():
            reference_quest_step(ops, qf, k, v, mins, maxs, p, c["topk"], c["sink_pages"], group)
        return reference, "reference", (
            f"{n_seq} of 16 sequences per step through the reference's torch operators (page_select_torch with the "
            f"sink forced, GQA union, block_sparse_attention_torch), fp32 on contiguous K/V, {threads} threads")
    ora = ctypes.CDLL(str(ROOT / "oracle" / "_build" / "liboracle.so"))
    ora.oracle_quest_decode.restype = ctypes.c_int
    to_bits = lambda x: x.to(torch.bfloat16).view(torch.int16).numpy()  # noqa: E731
    kb = to_bits(kp)
    vb = to_bits(vp)
    mn = to_bits(cache.meta_min[:n_seq].transpose(1, 2).contiguous().float().cpu())
    mx = to_bits(cache.meta_max[:n_seq].transpose(1, 2).contiguous().float().cpu())
    qh = to_bits(qf[:, :, 0].contiguous())
    table = np.arange(n_seq * n_pages, dtype=np.int32).reshape(n_seq, n_pages)
    lens = np.full(n_seq, t, dtype=np.int32)
    max_union = min(group * c["topk"], n_pages)
    out = np.zeros((n_seq, hq, d), dtype=np.float32)
    uids = np.zeros((n_seq, hkv, max_union), dtype=np.int32)
    ucnt = np.zeros((n_seq, hkv), dtype=np.int32)
    P_ = ctypes.c_void_p
    pool = ThreadPoolExecutor(threads)

    def run_unit(u):
        return ora.oracle_quest_decode(2, P_(qh.ctypes.data), P_(kb.ctypes.data), P_(vb.ctypes.data),
                                       P_(mn.ctypes.data), P_(mx.ctypes.data), P_(table.ctypes.data),
                                       P_(lens.ctypes.data), n_seq, hq, hkv, d, p, n_pages, c["topk"],
                                       c["sink_pages"], ctypes.c_float(1.0 / math.sqrt(d)), P_(out.ctypes.data),
                                       P_(uids.ctypes.data), P_(ucnt.ctypes.data), max_union, u, u + 1)

    def port():
        list(pool.map(run_unit, range(n_seq * hkv)))
    return port, "port", (f"{n_seq} of 16 sequences per step, selection + attention in the C oracle "
                          f"(oracle/c/oracle.c), {threads} threads")


def time_cpu(fn, min_seconds: float, max_iters: int = 1000):
    fn()  # warm
    t0 = time.perf_counter()
    n = 0
    while n < max_iters:
        fn()
        n += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    return (time.perf_counter() - t0) / n, n


# ---------------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    from linattn_b200 import QuestDecoder

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    c = C2
    b, hq, hkv, d, t, p = args.batch, c["Hq"], c["Hkv"], c["D"], c["T"], c["P"]
    n_q = args.warmup + args.steps
    cache, qs = build_c2(device, 1234 + rank, n_q, b)
    dec = QuestDecoder(cache, hq, c["topk"], sink_pages=c["sink_pages"], q_dtype=torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    for i in range(args.warmup):
        l2_flush(flush)
        dec.step(qs[i])
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    tokens = torch.zeros(args.steps, dtype=torch.int64, device=device)
    counts = torch.zeros(args.steps, dtype=torch.int64, device=device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys_gpu = int(visible.split(",")[local_rank]) if visible else local_rank
    with ClockSampler(phys_gpu) as clocks:
        t_wall = time.perf_counter()
        for i in range(args.steps):
            q = qs[args.warmup + i]
            l2_flush(flush)
            ev[i][0].record(stream)
            dec.select(q)
            ev[i][1].record(stream)
            dec.attend(q)
            ev[i][2].record(stream)
            tokens[i] = dec.union_tokens.sum()
            counts[i] = dec.union_count.sum()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        wall_s = time.perf_counter() - t_wall
    step_ms = [ev[i][0].elapsed_time(ev[i][2]) for i in range(args.steps)]
    sel_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
    att_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]
    mean_step = statistics.mean(step_ms)
    mean_sel = statistics.mean(sel_ms)
    mean_att = statistics.mean(att_ms)
    tok = tokens.float().mean().item()
    pages_sel = counts.float().mean().item()

    # ---- end to end through the public API: pinned host q -> step -> pinned host o
    q_host = qs.cpu().pin_memory()
    o_host = torch.empty((b, hq, 1, d), dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty_like(qs[0])
    e2e_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.warmup):
        q_dev.copy_(q_host[i], non_blocking=True)
        o_host.copy_(dec.step(q_dev), non_blocking=True)
    torch.cuda.synchronize(device)
    for i in range(args.steps):
        l2_flush(flush)
        e2e_ev[i][0].record(stream)
        q_dev.copy_(q_host[args.warmup + i], non_blocking=True)
        out = dec.step(q_dev)
        o_host.copy_(out, non_blocking=True)
        e2e_ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    e2e_eager_ms = statistics.mean(e.elapsed_time(f) for e, f in e2e_ev)
    # the same step as one CUDA graph (QuestDecoder.graph: pinned q in, pinned o out);
    # a serving loop reads o before it stages the next q, so every step is waited for
    g = dec.graph()
    for i in range(args.warmup):
        g.run(q_host[i])
        torch.cuda.synchronize(device)
    g_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        l2_flush(flush)
        g_ev[i][0].record(stream)
        g.run(q_host[args.warmup + i])
        g_ev[i][1].record(stream)
        g_ev[i][1].synchronize()
    e2e_ms = statistics.mean(e.elapsed_time(f) for e, f in g_ev)
    del g

    # ---- the resident step (selection + attention) replayed as one CUDA graph, as a
    # serving loop runs it; the eager per-phase events above give its breakdown
    q_static = qs[args.warmup].clone()
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        dec.select(q_static)
        dec.attend(q_static)
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    gstep = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gstep):
        dec.select(q_static)
        dec.attend(q_static)
    for i in range(args.warmup):
        q_static.copy_(qs[i])
        gstep.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    s_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        q_static.copy_(qs[args.warmup + i])
        l2_flush(flush)
        s_ev[i][0].record(stream)
        gstep.replay()
        s_ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    graph_step_ms = statistics.mean(e.elapsed_time(f) for e, f in s_ev)
    del gstep

    # ---- max over ranks
    vals = torch.tensor([mean_step, e2e_ms, mean_att, wall_s, e2e_eager_ms, graph_step_ms], dtype=torch.float64,
                        device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    mean_step, e2e_ms, mean_att_max, wall_s, e2e_eager_ms, graph_step_ms = vals.tolist()
    eager_step = mean_step
    mean_step = graph_step_ms

    elt = 2
    kv_bytes = tok * d * 2 * elt  # K and V rows actually read (union tokens)
    qo_bytes = 2 * b * hq * d * elt
    meta_bytes = 2 * b * hkv * (t // p) * d * elt
    score_bytes = 0 if dec.fused else 2 * b * hq * (t // p) * 4  # the fused selection keeps scores on chip
    if dec.fused and dec.chunks > 1:
        score_bytes = 2 * dec.cand.numel() * 4  # candidates written by the chunk CTAs, read by the merge
    step_bytes = kv_bytes + qo_bytes + meta_bytes + score_bytes
    hbm_peak, _, peak_kind = measured_peaks()
    att_bytes = kv_bytes + qo_bytes
    achieved_att = att_bytes / (mean_att * 1e-3) / 1e9
    traffic, traffic_info = profile_traffic("sparse_attention_c2.md")
    # this library's kernels per step: selection (fused, or candidates + merge), attention, split merge
    n_launch_step = (2 if dec.fused and dec.chunks > 1 else 1 if dec.fused else 2) + 1 + (1 if dec.n_splits > 1 else 0)
    clock = clocks.summary()
    line = {
        "metric": METRIC,
        "value": round(b * world / (mean_step * 1e-3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(mean_step, 4),
        "timing": "the step (selection + attention) replayed as one CUDA graph, L2 flushed before each, max over ranks",
        "eager_ms_per_step": round(eager_step, 4),
        "eager_value": round(b * world / (eager_step * 1e-3), 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 KV, 1% needle pages, random page-table permutation)",
        "config": {"workload": "quest_decode_c2" if b == C2["B"] else f"quest_decode_c2_b{b}", "batch_per_gpu": b, "global_batch": b * world, "seq_len": t,
                   "page_size": p, "n_heads": hq, "n_kv_heads": hkv, "head_dim": d,
                   "budget_pages": c["topk"], "sink_pages": c["sink_pages"], "parallelism": f"dp{world} (batch)",
                   "l2": L2_NOTE,
                   "n_splits": dec.n_splits, "select_chunks": dec.chunks},
        "hbm_gbs": round(step_bytes / (mean_step * 1e-3) / 1e9, 1),
        "step_breakdown_ms": {"select": round(mean_sel, 4), "attend": round(mean_att, 4)},
        "bytes_per_step": {"kv_union": int(kv_bytes), "meta": meta_bytes, "scores": score_bytes, "q_o": qo_bytes},
        "pages_per_kv_head": round(pages_sel / (b * hkv), 2),
        "wall_ms_per_step": round(wall_s * 1e3 / args.steps, 4),
        "roofline": {"bound": "hbm", "kernel": "sparse_attention (split-KV + merge)",
                     "achieved": round(achieved_att, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved_att / hbm_peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "traffic_source": traffic_info,
                     "algorithmic_bytes_per_launch": int(att_bytes)},
        "e2e": {"value": round(b * world / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(qs[0].numel() * elt), "d2h_bytes_per_step": int(o_host.numel() * elt),
                "ms_per_step": round(e2e_ms, 4), "api": "linattn_b200.QuestDecoder.graph().run (CUDA graph)",
                "eager_ms_per_step": round(e2e_eager_ms, 4),
                "eager_value": round(b * world / (e2e_eager_ms * 1e-3), 1)},
        "gpu_launches": n_launch_step * args.steps,
        "clocks": clock,
    }
    if world == 1 and not args.no_parity:
        line["parity"] = {"quest_decode_c2": parity_quest_decode(cache, qs[args.warmup], c["topk"], c["sink_pages"],
                                                                 n_splits=dec.n_splits,
                                                                 timed_out=dec.step(qs[args.warmup]).clone())}
    if world == 1 and not args.no_secondary:
        sec_steps, sec_warm = max(3, min(args.steps, 10)), 3

        def guarded(fn):
            # a secondary leg that fails reports its error; the headline line stands
            try:
                return fn(device, sec_steps, sec_warm, flush, stream)
            except Exception as exc:  # noqa: BLE001
                torch.cuda.synchronize(device)
                return {"error": f"{type(exc).__name__}: {exc}"[:300]}
        c4 = guarded(secondary_c4)
        if "prefill_tflops" in c4:
            line["prefill_tflops"] = c4["prefill_tflops"]
        torch.cuda.empty_cache()
        c3 = guarded(secondary_c3)
        line["secondary"] = {"block_sparse_prefill_c4": c4, "dsa_c3": c3}
        for key, r in (("block_sparse_prefill_c4", c4), ("dsa_c3", c3)):
            if "parity" in r:
                line.setdefault("parity", {})[key] = r.pop("parity")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        fn, kind, desc = cpu_reference_step_fn(cache, qs[args.warmup], 2, threads)
        sec, iters = time_cpu(fn, args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(2 / sec, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                                "sample": desc + f"; {iters} timed iterations of {sec * 1e3:.1f} ms"}
    return line


def run_c5(args, rank, world, local_rank):
    """Config 5: million-token decode with the KV sequence split over the ranks (strong
    scaling): local fused selection -> all-gather of (score, page) candidates -> global
    top-k + owned GQA union -> fp32 partial attention -> all-gather of [o | lse] ->
    log-sum-exp combine.  Both exchanges are NCCL all-gathers over NVLink (N > 1)."""
    from linattn_b200.sharded import ShardedQuestDecoder, exchange_packed

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    c = C5
    b, hq, hkv, d, t, p = args.batch or c["B"], c["Hq"], c["Hkv"], c["D"], args.seq_len or c["T"], c["P"]
    n_q = args.warmup + args.steps
    t_build = time.perf_counter()
    cache, qs, (lo, hi) = build_c5(device, rank, world, n_q, b, t)
    torch.cuda.synchronize(device)
    build_s = time.perf_counter() - t_build
    n_glob = t // p
    dec = ShardedQuestDecoder(cache, hq, c["topk"], [lo] * b, [hi] * b, last_here=(hi == n_glob),
                              sink_here=(lo == 0))
    exchange = (lambda x: exchange_packed(x)) if world > 1 else (lambda x: x.unsqueeze(0))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    box = {}

    def phase_select():
        dec.candidates(box["q"])

    def phase_merge():
        dec.merge_packed(exchange(dec.exchange_buf))

    def phase_attend():
        dec.partial(box["q"])

    def phase_combine():
        dec.combine_packed(exchange(dec.part))

    phases = [phase_select, phase_merge, phase_attend, phase_combine]
    for i in range(args.warmup):
        box["q"] = qs[i]
        l2_flush(flush)
        for f in phases:
            f()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(phases) + 1)] for _ in range(args.steps)]
    union_pages = torch.zeros(args.steps, dtype=torch.int64, device=device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys_gpu = int(visible.split(",")[local_rank]) if visible else local_rank
    with ClockSampler(phys_gpu) as clocks:
        t_wall = time.perf_counter()
        for i in range(args.steps):
            box["q"] = qs[args.warmup + i]
            l2_flush(flush)
            ev[i][0].record(stream)
            for j, f in enumerate(phases):
                f()
                ev[i][j + 1].record(stream)
            union_pages[i] = dec.union_count.sum()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        wall_s = time.perf_counter() - t_wall
    ph = [statistics.mean(ev[i][j].elapsed_time(ev[i][j + 1]) for i in range(args.steps)) for j in range(len(phases))]
    step_ms = statistics.mean(ev[i][0].elapsed_time(ev[i][-1]) for i in range(args.steps))
    pages_loc = union_pages.float().mean().item()

    # ---- end to end through the public API: pinned host q -> ShardedQuestDecoder.step -> pinned host o
    q_host = qs.cpu().pin_memory()
    o_host = torch.empty((b, hq, 1, d), dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty_like(qs[0])
    for i in range(args.warmup):
        q_dev.copy_(q_host[i], non_blocking=True)
        o_host.copy_(dec.step(q_dev, exchange=exchange), non_blocking=True)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    e2e_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        l2_flush(flush)
        e2e_ev[i][0].record(stream)
        q_dev.copy_(q_host[args.warmup + i], non_blocking=True)
        o_host.copy_(dec.step(q_dev, exchange=exchange), non_blocking=True)
        e2e_ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = statistics.mean(e.elapsed_time(f) for e, f in e2e_ev)

    # ---- the same step as one CUDA graph (the NCCL all-gathers captured with it): the
    # eager phases above carry the host's launch overhead between short kernels; a
    # serving loop replays the graph.  Pinned q in, pinned o out, every step waited for.
    graph_ms, graph_e2e_ms, graph_note = None, None, "captured"
    q_static = torch.empty_like(qs[0])
    g = None
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for i in range(2):
                q_static.copy_(qs[i])
                dec.step(q_static, exchange=exchange)
        stream.wait_stream(side)
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out_static = dec.step(q_static, exchange=exchange)
        torch.cuda.synchronize(device)
    except Exception as exc:  # noqa: BLE001  (the eager numbers stand)
        g, graph_note = None, f"not captured: {type(exc).__name__}: {exc}"[:200]
    if g is not None:
        for i in range(args.warmup):
            q_static.copy_(qs[i])
            g.replay()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        gev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        for i in range(args.steps):
            q_static.copy_(qs[args.warmup + i])
            l2_flush(flush)
            gev[i][0].record(stream)
            g.replay()
            gev[i][1].record(stream)
        torch.cuda.synchronize(device)
        graph_ms = statistics.mean(e.elapsed_time(f) for e, f in gev)
        if world > 1:
            torch.distributed.barrier()
        for i in range(args.steps):
            l2_flush(flush)
            gev[i][0].record(stream)
            q_static.copy_(q_host[args.warmup + i], non_blocking=True)
            g.replay()
            o_host.copy_(out_static, non_blocking=True)
            gev[i][1].record(stream)
            gev[i][1].synchronize()
        graph_e2e_ms = statistics.mean(e.elapsed_time(f) for e, f in gev)
        torch.cuda.synchronize(device)
        del g  # graphs holding NCCL calls go before the process group does
    gvals = torch.tensor([graph_ms or 0.0, graph_e2e_ms or 0.0, 0.0 if graph_ms is None else 1.0],
                         dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(gvals, op=torch.distributed.ReduceOp.MAX)
        ok_all = torch.tensor([0.0 if graph_ms is None else 1.0], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(ok_all, op=torch.distributed.ReduceOp.MIN)
        if ok_all.item() < 1.0:
            graph_ms = None
    if graph_ms is not None:
        graph_ms, graph_e2e_ms = gvals[0].item(), gvals[1].item()

    par = None
    if world == 1 and not args.no_parity:
        q_chk = qs[args.warmup]
        timed = dec.step(q_chk, exchange=exchange).clone()
        par = parity_quest_decode(cache, q_chk, c["topk"], 0, n_splits=dec.n_splits, timed_out=timed, tol=TOL_FP8)
    n_loc = hi - lo
    meta_bytes = b * hkv * n_loc * 2 * d * 2
    score_bytes = 0  # the fused kernel keeps page scores on chip; candidates are (chunks, B, H_q, topk)
    sel_bytes = meta_bytes + dec.cand.numel() * 4 * (2 if dec.premerge else 1)
    # per selected (page, kv head): fp8 K and V rows and their two fp32 scales; plus q in and f32 (o, lse) out
    kv_bytes = pages_loc * (p * d * 2 + 8) + b * hq * d * 2 + b * hq * (d + 1) * 4
    achieved_sel = sel_bytes / (ph[0] * 1e-3) / 1e9
    achieved_att = kv_bytes / (ph[2] * 1e-3) / 1e9
    vals = torch.tensor([step_ms, e2e_ms, wall_s, *ph, achieved_sel, achieved_att, build_s], dtype=torch.float64,
                        device=device)
    mins = vals.clone()
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(mins, op=torch.distributed.ReduceOp.MIN)
    step_ms, e2e_ms, wall_s, *rest = vals.tolist()
    ph_max, build_max = rest[:4], rest[6]
    sel_min_gbs, att_min_gbs = mins[7].item(), mins[8].item()
    hbm_peak, _, peak_kind = measured_peaks()
    dominant = "select" if ph[0] >= ph[2] else "attend"
    ach = sel_min_gbs if dominant == "select" else att_min_gbs
    kname = "quest_decode_candidates (fused page scoring + per-chunk top-k)" if dominant == "select" else \
        "sparse_attention (fp8 paged on tensor cores, f32 partial o + lse)"
    traffic, traffic_info = profile_traffic("quest_select_c5.md" if dominant == "select" else "sparse_attention_c5.md")
    # candidates (+ the shard's pre-merge), merge, attention (+ its split merge), combine
    n_mine = 4 + (dec.n_splits > 1) + int(dec.premerge)
    eager_step_ms, eager_e2e_ms = step_ms, e2e_ms
    if graph_ms is not None:
        step_ms, e2e_ms = graph_ms, graph_e2e_ms
    return {
        "metric": METRIC,
        "value": round(b / (step_ms * 1e-3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "timing": ("the step replayed as one CUDA graph (NCCL all-gathers inside), max over ranks"
                   if graph_ms is not None else "eager launches, max over ranks") + f"; graph {graph_note}",
        "eager_ms_per_step": round(eager_step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8e4m3 KV, bf16 q, f32 accumulate",
        "data": "synthetic (seeded N(0,1) values quantised to e4m3 per (page, kv head), 0.5% needle pages at "
                "global positions shared by every rank, random page table per shard)",
        "config": {"workload": "sharded_decode_c5" if (b, t) == (C5["B"], C5["T"]) else f"sharded_decode_c5_b{b}_t{t}",
                   "batch": b,
                   "seq_len": t, "page_size": p, "n_heads": hq, "n_kv_heads": hkv, "head_dim": d,
                   "budget_pages": c["topk"], "pages_per_gpu_per_seq": n_loc,
                   "parallelism": f"sequence-sharded x{world} (KV pages split, NCCL all-gathers)",
                   "l2": L2_NOTE + "; per-step inputs (page metadata + selected pages) exceed L2 anyway"},
        "step_breakdown_ms": {"select": round(ph_max[0], 4), "exchange_candidates+merge": round(ph_max[1], 4),
                              "attend": round(ph_max[2], 4), "exchange_partials+combine": round(ph_max[3], 4)},
        "bytes_per_step_per_gpu": {"meta": int(meta_bytes), "scores": int(score_bytes), "kv_selected": int(kv_bytes)},
        "selected_pages_per_kv_head_per_gpu": round(pages_loc / (b * hkv), 2),
        "select_chunks_per_gpu": dec.chunks, "pages_per_select_cta": dec.chunk_pages, "attend_splits": dec.n_splits,
        "wall_ms_per_step": round(wall_s * 1e3 / args.steps, 4),
        "build_s": round(build_max, 1),
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(ach / hbm_peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                     "traffic_source": traffic_info,
                     "algorithmic_bytes_per_launch": int(sel_bytes if dominant == "select" else kv_bytes),
                     "note": "slowest rank's achieved bandwidth"},
        "e2e": {"value": round(b / (e2e_ms * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": int(qs[0].numel() * 2),
                "d2h_bytes_per_step": int(o_host.numel() * 2), "ms_per_step": round(e2e_ms, 4),
                "api": "linattn_b200.sharded.ShardedQuestDecoder.step" + (
                    " captured as a CUDA graph" if graph_ms is not None else ""),
                "eager_ms_per_step": round(eager_e2e_ms, 4)},
        "gpu_launches": n_mine * args.steps,
        "clocks": clocks.summary(),
        **({"parity": {"sharded_decode_c5": par}} if par is not None else {}),
    }


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_bench_decode(threads: int):
    """The reference's ``bench/bench_decode.py`` as shipped (from its copy in
    ``baseline/_ref``; it pins min(4, threads) torch threads itself), its printed
    records parsed."""
    import subprocess

    script = REF_DIR / "bench" / "bench_decode.py"
    if not script.exists():
        return {"unavailable": "baseline/_ref/bench/bench_decode.py not installed"}
    env = dict(os.environ, PYTHONPATH=str(REF_DIR), OMP_NUM_THREADS=str(threads))
    res = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, env=env, timeout=600)
    import re

    recs = []
    pat = re.compile(r"^(\S+)\s+entries=\s*(\d+)\s+bytes=\s*([\d.]+) MiB\s+([\d.]+) ms\s+([\d.]+) GiB/s")
    for line in res.stdout.splitlines():
        m = pat.match(line.strip())
        if m:
            recs.append({"policy": m.group(1), "kv_entries": int(m.group(2)), "mib": float(m.group(3)),
                         "ms": float(m.group(4)), "gib_s": float(m.group(5))})
    return {"cmd": "python bench/bench_decode.py (defaults: --seq 65536 --dim 64 --page 16 --budgets 256 1024 2048 "
                   "8192 --repeat 5)", "rc": res.returncode, "torch_threads": min(4, threads), "records": recs}


def run_reference(args):
    """Reference arm: the reference's own CPU torch path for the config-2 step on the
    host cores (all of them), over the whole config (16 sequences of 65536 tokens),
    with inputs built on the host; this library is not imported in this process."""
    ops = reference_ops()
    c = C2
    threads = os.cpu_count() or 1
    if ops is None:
        return {"impl": "reference", "unavailable": "the reference is not installed in baseline/_ref"}
    torch.set_num_threads(threads)
    t_build = time.perf_counter()
    k, v, qs = build_c2_host(1234, args.warmup + args.steps, c["B"], threads)
    mins, maxs = ops[0](k, c["P"])  # maintained on append in a serving loop: outside the step
    build_s = time.perf_counter() - t_build
    group = c["Hq"] // c["Hkv"]

    def step(i):
        return reference_quest_step(ops, qs[i], k, v, mins, maxs, c["P"], c["topk"], c["sink_pages"], group)
    for i in range(args.warmup):
        step(i)
    times = []
    pages = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        _, union = step(args.warmup + i)
        times.append(time.perf_counter() - t0)
        pages.append(float(union.sum()) / (c["B"] * c["Hkv"]))
    sec = statistics.mean(times)
    value = c["B"] / sec
    desc = (f"the whole config-2 step (16 sequences) per timed step through the reference's torch operators: "
            f"page_select_torch (own page forced, sink page forced in its place), the GQA union, "
            f"block_sparse_attention_torch; fp32 on contiguous K/V holding bf16 values; {threads} torch threads")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 (bf16 values widened exactly)",
        "data": "synthetic, built on the host: the CUDA arm's construction (N(0,1) bf16 K/V, 1% needle pages, "
                "queries around a base query) from numpy generators; contiguous layout (the reference has no page "
                "table)",
        "config": {"workload": "quest_decode_c2", "batch_per_gpu": c["B"], "global_batch": c["B"], "seq_len": c["T"],
                   "page_size": c["P"], "n_heads": c["Hq"], "n_kv_heads": c["Hkv"], "head_dim": c["D"],
                   "budget_pages": c["topk"], "sink_pages": c["sink_pages"], "parallelism": "host cores"},
        "pages_per_kv_head": round(statistics.mean(pages), 2),
        "build_s": round(build_s, 1),
        "host": {"cpu": _cpu_model(), "cores": threads, "torch_threads": torch.get_num_threads()},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads,
                         "kind": "reference (torch: page_select_torch + block_sparse_attention_torch)",
                         "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "bench_decode_as_shipped": reference_bench_decode(threads),
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (default: the config's; smaller only for profiling captures)")
    ap.add_argument("--workload", default="c2", choices=["c2", "c3", "c4", "c5", "variants"],
                    help="c2: paged Quest decode (the headline); c3: DSA indexer + token attention; c4: block-sparse "
                         "prefill; c5: million-token sequence-sharded decode; variants: the CSA2 and NSA plugins' "
                         "prefill forward")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="c3 / c4 / c5 only: a shorter sequence (profiling captures)")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the full-size parity checks (run outside the timed regions)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config-3 / config-4 legs reported beside the config-2 line")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.workload != "c2":
            print(json.dumps({"impl": "reference", "unavailable": "the reference's CPU arm is timed on the config-2 "
                              "workload (its torch paths for configs 3-5 need O(T^2) masks or more host memory than "
                              "this box has)"}), flush=True)
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0
    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "c5":
            line = run_c5(args, rank, world, local_rank)
        elif args.workload in ("c3", "c4"):
            if world > 1:
                raise SystemExit("--workload c3 / c4 run on one GPU")
            line = run_prefill_workload(args)
        elif args.workload == "variants":
            if world > 1:
                raise SystemExit("--workload variants runs on one GPU")
            line = run_variants_workload(args)
        else:
            if args.batch is None:
                args.batch = C2["B"]
            line = run_ours(args, rank, world, local_rank)
            if not args.no_secondary:
                # config 5 beside the headline at every N: the KV sequence split over the
                # ranks (strong scaling), the one configuration with a data-path collective
                torch.cuda.empty_cache()
                c5_args = argparse.Namespace(**vars(args))
                c5_args.batch, c5_args.seq_len = None, None
                c5_args.steps, c5_args.warmup = max(3, min(args.steps, 10)), 3
                try:
                    c5 = run_c5(c5_args, rank, world, local_rank)
                except Exception as exc:  # noqa: BLE001  (the headline line stands)
                    c5 = {"error": f"{type(exc).__name__}: {exc}"[:300]}
                if rank == 0 and "error" in c5:
                    line.setdefault("secondary", {})["sharded_decode_c5"] = c5
                elif rank == 0:
                    keep = ("value", "unit", "n_gpus", "ms_per_step", "timing", "eager_ms_per_step", "scaling", "dtype",
                            "config",
                            "step_breakdown_ms", "bytes_per_step_per_gpu", "selected_pages_per_kv_head_per_gpu",
                            "select_chunks_per_gpu", "attend_splits", "roofline", "e2e", "gpu_launches", "clocks")
                    line.setdefault("secondary", {})["sharded_decode_c5"] = {k: c5[k] for k in keep if k in c5}
                    if "parity" in c5:
                        line.setdefault("parity", {}).update(c5["parity"])
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
