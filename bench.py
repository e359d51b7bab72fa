#!/usr/bin/env python
"""Benchmark of the sparse-attention hot path on B200.

Workload ("quest_decode_c2"): paged Quest decode, one new token for each of B=16
sequences per GPU, H_q=32, H_kv=8, D=128, T=65536 per sequence in pages of 64
(1024 pages), bf16 KV with 1% needle pages along each kv group's query direction,
pages scattered by a seeded random permutation over a pool of 16x1024 pages; budget
32 pages + sink page 0 + the last page per query head (top-34 with both forced),
GQA union per kv head.  A step = page scoring + top-k/union + sparse attention
(split-KV + merge) for all 16 sequences; inputs resident in HBM, L2 flushed (a
256 MiB write) before every step, outside the timed events.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
prints one JSON line.  For N > 1 (torchrun) every rank runs its own 16 sequences
(weak scaling, no data-path collective) and the step time is the max over ranks.
``--impl reference`` times the reference's CPU path on the host cores (rank 0 only).
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
L2_FLUSH_BYTES = 256 << 20


# ---------------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------------
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


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


# ---------------------------------------------------------------------------------
# CPU baselines (rank 0, N == 1 / reference arm): bounded samples of the workload
# ---------------------------------------------------------------------------------
def _cpu_sample(cache, q, n_seq: int):
    """Host copies of sequences [0, n_seq): contiguous logical pages, bf16 bits."""
    tab = cache.page_table[:n_seq].long()
    kp = cache.k_pool[tab.flatten()].view(torch.int16).cpu().numpy()  # (n_seq*n_pages, Hkv, P, D)
    vp = cache.v_pool[tab.flatten()].view(torch.int16).cpu().numpy()
    # metadata is stored per sequence in logical page order: (n_seq, H_kv, pages, D)
    mn = cache.meta_min[:n_seq].transpose(1, 2).contiguous().view(torch.int16).cpu().numpy()
    mx = cache.meta_max[:n_seq].transpose(1, 2).contiguous().view(torch.int16).cpu().numpy()
    qh = q[:n_seq, :, 0].contiguous().view(torch.int16).cpu().numpy()
    return kp, vp, mn, mx, qh


def cpu_reference_step_fn(cache, q, n_seq: int, threads: int):
    """Returns (fn, kind, description): fn() runs one CPU step over the sample.

    Selection = the oracle's C restatement (oracle/c/oracle.c, the reference's page
    selection is torch code); attention = the reference's own C kernel
    ``paged_decode_tiled`` (src/linattn/kernels/c/decode_attn.c:72-133, compiled to
    oracle/_ref) over each query head's union pages on fp32 contiguous K/V, the
    layout that kernel takes.  Without oracle/_ref the C oracle does both ("port").
    """
    c = C2
    hq, hkv, d, p, t = c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    n_pages = t // p
    group = hq // hkv
    kp, vp, mn, mx, qh = _cpu_sample(cache, q, n_seq)
    ora = ctypes.CDLL(str(ROOT / "oracle" / "_build" / "liboracle.so"))
    ora.oracle_quest_decode.restype = ctypes.c_int
    table = np.arange(n_seq * n_pages, dtype=np.int32).reshape(n_seq, n_pages)
    lens = np.full(n_seq, t, dtype=np.int32)
    max_union = min(group * c["topk"], n_pages)
    out = np.zeros((n_seq, hq, d), dtype=np.float32)
    uids = np.zeros((n_seq, hkv, max_union), dtype=np.int32)
    ucnt = np.zeros((n_seq, hkv), dtype=np.int32)
    scale = 1.0 / math.sqrt(d)
    P_ = ctypes.c_void_p

    def run_units(u0, u1):
        return ora.oracle_quest_decode(2, P_(qh.ctypes.data), P_(kp.ctypes.data), P_(vp.ctypes.data),
                                       P_(mn.ctypes.data), P_(mx.ctypes.data), P_(table.ctypes.data),
                                       P_(lens.ctypes.data), n_seq, hq, hkv, d, p, n_pages, c["topk"],
                                       c["sink_pages"], ctypes.c_float(scale), P_(out.ctypes.data),
                                       P_(uids.ctypes.data), P_(ucnt.ctypes.data), max_union, u0, u1)

    pool = ThreadPoolExecutor(threads)
    units = n_seq * hkv
    ref_lib = ROOT / "oracle" / "_ref" / "libdecode_attn.so"
    if not ref_lib.exists():
        def port():
            list(pool.map(lambda u: run_units(u, u + 1), range(units)))
        return port, "port", (f"{n_seq} of 16 sequences per step, full selection + attention in the C oracle "
                              f"(oracle/c/oracle.c), {threads} threads")
    ref = ctypes.CDLL(str(ref_lib))
    f32p = ctypes.POINTER(ctypes.c_float)
    i32p = ctypes.POINTER(ctypes.c_int32)
    ref.paged_decode_tiled.argtypes = [f32p, f32p, f32p, i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, f32p]
    # the reference kernel's storage: fp32 contiguous (T, D) per (sequence, kv head)
    def bf16_to_f32(a):
        return (a.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)

    kf = bf16_to_f32(kp).reshape(n_seq, n_pages, hkv, p, d).transpose(0, 2, 1, 3, 4).reshape(n_seq, hkv, t, d).copy()
    vf = bf16_to_f32(vp).reshape(n_seq, n_pages, hkv, p, d).transpose(0, 2, 1, 3, 4).reshape(n_seq, hkv, t, d).copy()
    qf = bf16_to_f32(qh).reshape(n_seq, hq, d).copy()
    out_ref = np.zeros((n_seq, hq, d), dtype=np.float32)

    def ref_head(idx):
        bi, h = divmod(idx, hq)
        kh = h // group
        ids = np.ascontiguousarray(uids[bi, kh, : ucnt[bi, kh]])
        ref.paged_decode_tiled(qf[bi, h].ctypes.data_as(f32p), kf[bi, kh].ctypes.data_as(f32p),
                               vf[bi, kh].ctypes.data_as(f32p), ids.ctypes.data_as(i32p), int(ids.size), p, d, t,
                               ctypes.c_float(scale), out_ref[bi, h].ctypes.data_as(f32p))

    ora.oracle_quest_select.restype = ctypes.c_int

    def select_units(u0, u1):
        return ora.oracle_quest_select(2, P_(qh.ctypes.data), P_(mn.ctypes.data), P_(mx.ctypes.data),
                                       P_(table.ctypes.data), P_(lens.ctypes.data), n_seq, hq, hkv, d, p, n_pages,
                                       c["topk"], c["sink_pages"], P_(uids.ctypes.data), P_(ucnt.ctypes.data),
                                       max_union, u0, u1)

    def reference():
        list(pool.map(lambda u: select_units(u, u + 1), range(units)))  # page selection (C oracle)
        list(pool.map(ref_head, range(n_seq * hq)))                      # the reference's C decode kernel

    return reference, "reference", (
        f"{n_seq} of 16 sequences per step; page selection in the C oracle (oracle/c/oracle.c, the reference's "
        f"selection is torch code) and attention with the reference's own paged_decode_tiled (decode_attn.c, "
        f"compiled from the reference source into oracle/_ref) on fp32 contiguous K/V, one call per query head; "
        f"{threads} threads")


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
        flush.zero_()
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
            flush.zero_()
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
        flush.zero_()
        e2e_ev[i][0].record(stream)
        q_dev.copy_(q_host[args.warmup + i], non_blocking=True)
        out = dec.step(q_dev)
        o_host.copy_(out, non_blocking=True)
        e2e_ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = statistics.mean(e.elapsed_time(f) for e, f in e2e_ev)

    # ---- max over ranks
    vals = torch.tensor([mean_step, e2e_ms, mean_att, wall_s], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    mean_step, e2e_ms, mean_att_max, wall_s = vals.tolist()

    elt = 2
    kv_bytes = tok * d * 2 * elt  # K and V rows actually read (union tokens)
    qo_bytes = 2 * b * hq * d * elt
    meta_bytes = 2 * b * hkv * (t // p) * d * elt
    score_bytes = 0 if dec.fused else 2 * b * hq * (t // p) * 4  # the fused selection keeps scores on chip
    step_bytes = kv_bytes + qo_bytes + meta_bytes + score_bytes
    hbm_peak, _, peak_kind = measured_peaks()
    att_bytes = kv_bytes + qo_bytes
    achieved_att = att_bytes / (mean_att * 1e-3) / 1e9
    traffic = profile_traffic("sparse_attention_c2.md")
    n_launch_step = 3 + (1 if dec.n_splits > 1 else 0)
    clock = clocks.summary()
    line = {
        "metric": METRIC,
        "value": round(b * world / (mean_step * 1e-3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(mean_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 KV, 1% needle pages, random page-table permutation)",
        "config": {"workload": "quest_decode_c2" if b == C2["B"] else f"quest_decode_c2_b{b}", "batch_per_gpu": b, "global_batch": b * world, "seq_len": t,
                   "page_size": p, "n_heads": hq, "n_kv_heads": hkv, "head_dim": d,
                   "budget_pages": c["topk"], "sink_pages": c["sink_pages"], "parallelism": f"dp{world} (batch)",
                   "l2": "flushed (256 MiB write) before every step, outside the timed events",
                   "n_splits": dec.n_splits},
        "hbm_gbs": round(step_bytes / (mean_step * 1e-3) / 1e9, 1),
        "step_breakdown_ms": {"select": round(mean_sel, 4), "attend": round(mean_att, 4)},
        "bytes_per_step": {"kv_union": int(kv_bytes), "meta": meta_bytes, "scores": score_bytes, "q_o": qo_bytes},
        "pages_per_kv_head": round(pages_sel / (b * hkv), 2),
        "wall_ms_per_step": round(wall_s * 1e3 / args.steps, 4),
        "roofline": {"bound": "hbm", "kernel": "sparse_attention (split-KV + merge)",
                     "achieved": round(achieved_att, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved_att / hbm_peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": int(att_bytes)},
        "e2e": {"value": round(b * world / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(qs[0].numel() * elt), "d2h_bytes_per_step": int(o_host.numel() * elt),
                "ms_per_step": round(e2e_ms, 4), "api": "linattn_b200.QuestDecoder.step"},
        "gpu_launches": n_launch_step * args.steps,
        "clocks": clock,
        "prefill_tflops": None,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        fn, kind, desc = cpu_reference_step_fn(cache, qs[args.warmup], 2, threads)
        sec, iters = time_cpu(fn, args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(2 / sec, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                                "sample": desc + f"; {iters} timed iterations of {sec * 1e3:.1f} ms"}
    return line


def run_reference(args):
    """Reference arm: the reference's CPU path on the host cores, bounded samples."""
    device = torch.device("cuda", 0)
    c = C2
    cache, qs = build_c2(device, 1234, args.warmup + args.steps)
    threads = os.cpu_count() or 1
    n_seq = 2
    fn, kind, desc = cpu_reference_step_fn(cache, qs[0], n_seq, threads)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    sec = (time.perf_counter() - t0) / args.steps
    value = n_seq / sec
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
        "dtype": "bf16",
        "data": "synthetic (same generator and seed as the CUDA arm)",
        "config": {"workload": "quest_decode_c2", "batch_per_gpu": c["B"], "seq_len": c["T"], "page_size": c["P"],
                   "n_heads": c["Hq"], "n_kv_heads": c["Hkv"], "head_dim": c["D"], "budget_pages": c["topk"],
                   "sample_sequences_per_step": n_seq},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=C2["B"],
                    help="sequences per GPU (16 = config 2; smaller only for profiling captures)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0
    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
