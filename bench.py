#!/usr/bin/env python3
"""Benchmark of the paged-KV hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl reference]

Default workload: BASELINE config 3, the config the metric's 1/2/4/8-GPU reading is quoted on --
one decode step of 256 sequences with lognormal context lengths (median 1500, sigma 1, clipped to
16..32768) whose block tables come from a seeded 10k-operation admit/evict churn of a 65536-block
pool (28 query / 4 kv heads, d 128, fp32 KV, 16-token blocks).  The 256 sequences are ONE global
batch split over the GPUs by longest-first partitioning (strong scaling): every rank owns a pool
and decodes its share, with no collective.  A "step" is: upload the step's tables (one host-to-
device copy), decode every sequence; tokens/s = sequences decoded per second.  cfg2 (append +
decode of 64 x 2048 tokens, weak-scaled), cfg1, cfg3-bf16, cfg4 (prefill), cfg5 (split-KV over
GPUs) and the append / copy kernels run with --config.

`value` times the step with inputs resident in HBM (CUDA events, max over ranks).  `e2e`
times the same iteration through gkv_decode_step_host with pinned HOST buffers (q, new K/V,
tables in; attention output out), every copy included, the last output copy too.

`--impl reference` times the CPU restatement of the reference's PagedAttentionKernel
(oracle/, faithful threading: sequences serial, OpenMP over query heads) on all host cores;
the reference itself is C# and cannot be built in this image.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "glacier.serve_b200"))

METRIC = "decode KV GB/s per B200 vs HBM peak; decode tokens/s at 1/2/4/8 GPUs vs C# CPU"
UNIT = "tokens/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# Configs whose sequences are one fixed global batch split over the GPUs (strong scaling):
# cfg3 by longest-first partitioning, cfg5 by block range.  cfg1 / cfg2 give every GPU its own
# batch (weak scaling).
STRONG = ("cfg3", "cfg3-bf16", "cfg3-f16", "cfg3-fp8", "cfg5")
CFG3 = {"cfg3": "f32", "cfg3-bf16": "bf16", "cfg3-f16": "f16", "cfg3-fp8": "fp8"}


def workload(name: str, rank: int, world: int = 1, batch: int = 0):
    """This rank's workload.  batch > 0 shrinks cfg2 / cfg3 to that many sequences (small cases
    for profiler captures)."""
    from glacier_kv import workloads as W

    seed = W.SEED + 1000003 * rank
    if name == "cfg1":
        return W.cfg1(seed)
    if name == "cfg2":
        return W.cfg2(seed, batch=batch or 64)
    if name in CFG3:  # the same 256 sequences everywhere, LPT share per rank
        w = W.cfg3(W.SEED, CFG3[name], batch=batch or 256)
        return w if world == 1 else W.lpt_share(w, rank, world)
    if name == "cfg5":  # this rank's block range of the 4 x 131072 sequences
        return W.cfg5_local(rank, world, W.SEED)
    raise SystemExit(f"unknown config {name}")


def describe(w) -> str:
    return (f"{w.name}: {'append+decode' if w.slot_mapping.size else 'decode'}, {w.batch} seqs, "
            f"sum ctx {int(w.ctx_lens.sum())} (max {int(w.ctx_lens.max())}), {w.n_heads}q/{w.heads_kv}kv heads, "
            f"d {w.head_dim}, {w.dtype} KV, block {w.block_size}, pool {w.total_blocks} blocks")


class Clocks:
    """Read-only NVML poller (SM clock, max clock, power, clock-event reasons) on a thread.

    Started before warm-up and stopped after the timed region; `mark()` opens and closes the
    timed window so the summary reports the samples taken inside it (plus one sample taken
    synchronously at each edge, so even a short window has data)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device):
        self.rows = []          # (t, sm_mhz, max_mhz, power_w, reasons_mask)
        self.window = [None, None]
        self.h = None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            p = torch.cuda.get_device_properties(device)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            self.h = None

    def sample(self):
        nv = self.nv
        try:
            sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
            mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.rows.append((time.perf_counter(), sm, mx, pw, rs))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(0.005)

    def __enter__(self):
        if self.h is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def mark(self, edge: int):
        if self.h is not None:
            self.sample()
            self.window[edge] = time.perf_counter()

    def __exit__(self, *exc):
        if self.h is not None:
            self._stop.set()
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled: NVML unavailable"]}
        lo, hi = self.window
        inside = [r for r in self.rows if lo is not None and hi is not None and lo <= r[0] <= hi]
        rows = inside or self.rows
        reasons = sorted({n for r in rows for n, m in self.REASONS.items() if r[4] & m})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(rows),
                "window": "timed region" if inside else "warm-up + timed region",
                "power_w_max": max(r[3] for r in rows)}


def traffic_from_profiles(cfg: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        d = json.load(open(p))
        e = d.get(cfg)
        if e:
            return e.get("dram_bytes_per_launch")
    return None


def cpu_baseline_run(w, steps: int, budget_s: float, threads: int, seed: int):
    """Times the CPU restatement (oracle/) of PagedAttentionKernel on a bounded sample of
    the workload: `sample` sequences with their real context lengths, arena restricted to
    their blocks, one sample per step."""
    from oracle import pyoracle as O

    rng = np.random.default_rng(seed)
    sample = min(w.batch, 16)
    rows = np.sort(rng.choice(w.batch, sample, replace=False))
    ctx = w.ctx_lens[rows]
    bs = w.block_size
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    tables = np.full((sample, max(nblk)), -1, np.int32)
    at = 0
    for i, n in enumerate(nblk):
        tables[i, :n] = np.arange(at, at + n, dtype=np.int32)
        at += n
    g = O.geom(at, 1, w.heads_kv, w.head_dim, w.v_head_dim, bs, {"f32": O.F32, "bf16": O.BF16, "f16": O.F16, "fp8": O.FP8}[w.dtype])
    K, V = O.new_arena(g)
    for arr in (K, V):
        arr[...] = O.to_storage_bits(rng.standard_normal(arr.shape, dtype=np.float32), g.dtype)
    q = rng.standard_normal((sample, w.n_heads, w.head_dim)).astype(np.float32)
    O.decode_batch(K, V, g, 0, tables, ctx, q, w.n_heads, w.scale, n_threads=threads)  # warm-up
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        O.decode_batch(K, V, g, 0, tables, ctx, q, w.n_heads, w.scale, n_threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    med = statistics.median(times)
    return {
        "value": sample / med,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": (f"{sample} of {w.batch} sequences of {w.name} (their real ctx lengths, "
                   f"{int(ctx.sum())} tokens), median of {len(times)} runs; sequences serial, "
                   f"OpenMP over query heads as PagedAttentionKernel.cs:48"),
        "ms_per_sample": med * 1e3,
    }


PREFILL_METRIC = "chunked causal prefill TFLOP/s (causal FLOP count) per B200 vs bf16 tensor peak"


def prefill_cpu_baseline(w, steps: int, budget_s: float, threads: int, seed: int, n_q: int = 24):
    """Times the CPU restatement (oracle/) of the reference's prefill (one ComputeAttention per
    chunk token, PagedTransformerRunner.cs:454-471) on a bounded sample: the last n_q queries of
    one sequence's chunk (the heaviest rows), arena restricted to that sequence's blocks."""
    from oracle import pyoracle as O

    rng = np.random.default_rng(seed)
    b = int(np.argmax(w.prefix))
    tok = int(w.token_counts[b])
    bs = w.block_size
    nblk = (tok + bs - 1) // bs
    g = O.geom(nblk, 1, w.heads_kv, w.head_dim, w.v_head_dim, bs, O.BF16)
    K, V = O.new_arena(g)
    for arr in (K, V):
        arr[...] = O.f32_to_bf16_bits(rng.standard_normal(arr.shape, dtype=np.float32))
    ids = np.arange(nblk, dtype=np.int32)
    q = rng.standard_normal((n_q, w.n_heads, w.head_dim)).astype(np.float32)
    start = tok - n_q
    O.prefill_chunk(K, V, g, 0, ids, tok, start, q, w.n_heads, w.scale, n_threads=threads)  # warm-up
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        O.prefill_chunk(K, V, g, 0, ids, tok, start, q, w.n_heads, w.scale, n_threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    med = statistics.median(times)
    flops = 2 * (w.head_dim + w.v_head_dim) * w.n_heads * sum(start + t + 1 for t in range(n_q))
    return {
        "value": flops / med / 1e12,
        "unit": "TFLOP/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"last {n_q} chunk queries of {w.name} sequence {b} (positions {start}..{tok - 1}), "
                   f"median of {len(times)} runs; one ComputeAttention per query, OpenMP over query heads"),
        "ms_per_sample": med * 1e3,
    }


def mapped_native_libs():
    """Shared objects of this repository mapped into the process (from /proc/self/maps)."""
    out = set()
    try:
        with open("/proc/self/maps") as f:
            for ln in f:
                path = ln.split()[-1] if len(ln.split()) >= 6 else ""
                if path.endswith(".so") and os.path.realpath(path).startswith(os.path.realpath(ROOT)):
                    out.add(os.path.relpath(os.path.realpath(path), os.path.realpath(ROOT)))
    except OSError:
        pass
    return sorted(out)


def run_reference(args):
    """The reference arm: the CPU restatement (oracle/) of the reference's own code for the path,
    timed on the host cores with the thread count passed explicitly (a torchrun launch sets
    OMP_NUM_THREADS=1, which must not shrink the baseline).  Maps no native code of the product:
    the workload generators are numpy only and glacier_kv's library loads on first use."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import pyoracle as O

    cores = O.host_cores()
    if args.config == "cfg4":
        from glacier_kv import workloads as W

        w = W.cfg4(W.SEED)
        res = prefill_cpu_baseline(w, max(args.steps, 1), budget_s=120.0, threads=cores, seed=w.seed)
        line = {
            "metric": PREFILL_METRIC, "value": res["value"], "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_sample"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": describe_prefill(w), "l2": "n/a (CPU)",
                       "implementation": "C restatement of PagedTransformerRunner.ForwardPrefillSubBatch + "
                                         "PagedAttentionKernel.ComputeAttention"},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    elif args.config in BANDWIDTH_CONFIGS:
        res = bandwidth_cpu_baseline(args.config, max(args.steps, 1), budget_s=120.0)
        line = {
            "metric": f"{bandwidth_metric(args.config)} GB/s per B200 vs HBM peak",
            "value": res["value"], "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_sample"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if args.config.endswith("bf16") else "f32",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": args.config, "l2": "n/a (CPU)",
                       "implementation": "C restatement of PagedBlockPool.Store / CopyBlockData and the runner loop "
                                         "(serial in the reference, so one thread)"},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    else:
        w = workload(args.config, 0)
        res = cpu_baseline_run(w, max(args.steps, 1), budget_s=120.0, threads=cores, seed=w.seed)
        line = {
            "metric": METRIC, "value": res["value"], "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_sample"], "higher_is_better": True,
            "scaling": "strong" if args.config in STRONG else "weak",
            "vs_baseline": None, "dtype": "f32", "kv_dtype": w.dtype, "data": "synthetic (seeded N(0,1))",
            "config": {"workload": describe(w), "l2": "n/a (CPU)",
                       "implementation": "C restatement of PagedAttentionKernel.ComputeAttention "
                                         "(the C# reference needs .NET 10 + un-vendored NuGet; not buildable here)"},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    line["host_cores"] = cores
    line["native_so_loaded"] = mapped_native_libs()
    print(json.dumps(line), flush=True)


def describe_prefill(w) -> str:
    return (f"{w.name}: append {w.chunk} tokens per sequence + chunked causal prefill, {w.batch} seqs, "
            f"prefixes {w.prefix.tolist()}, {w.n_heads}q/{w.heads_kv}kv heads, d {w.head_dim}, {w.dtype} Q/K/V, "
            f"fp32 softmax and output, block {w.block_size}, pool {w.total_blocks} blocks")


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    return 1590.0, "fallback 1.59 PFLOP/s"


def run_prefill(args, world, rank, local, dev, barrier, max_over_ranks):
    """cfg4: one step = upload tables + slots, append the 8 x 2048 chunk tokens, prefill them.
    Weak scaling: every rank owns a pool and its own 8 sequences."""
    import torch

    import glacier_kv as G
    from glacier_kv import workloads as W

    w = W.cfg4(W.SEED + 1000003 * rank)
    pool = G.PagedBlockPool(w.total_blocks, 1, w.heads_kv, w.head_dim, w.block_size, w.v_head_dim,
                            device=local, dtype=w.dtype)
    W.fill_arena_randn(pool, seed=w.seed)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(w.seed + 17)
    nq = w.n_queries
    q = torch.from_numpy(rng.standard_normal((nq, w.n_heads, w.head_dim), dtype=np.float32)).to(dev).to(torch.bfloat16)
    kn = torch.from_numpy(rng.standard_normal((nq, w.heads_kv, w.head_dim), dtype=np.float32)).to(dev)
    vn = torch.from_numpy(rng.standard_normal((nq, w.heads_kv, w.v_head_dim), dtype=np.float32)).to(dev)
    out = torch.empty((nq, w.n_heads, w.v_head_dim), dtype=torch.float32, device=dev)
    toks, qs, ql = w.token_counts, w.prefix.astype(np.int32), w.q_lens
    pool.reserve_step(w.batch, w.tables.shape[1], nq, w.n_heads)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def step(pre_ev=None):
        pool.upload_step(w.tables, toks, w.slot_mapping, stream=stream)
        pool.kv_append(0, kn, vn, stream=stream)
        n = pool.last_launch_count
        if pre_ev is not None:
            pre_ev[0].record(stream)
        pool.paged_prefill(0, q, out, qs, ql, w.n_heads, w.scale, stream=stream)
        if pre_ev is not None:
            pre_ev[1].record(stream)
        return n + pool.last_launch_count

    clk = Clocks(dev)
    clk.__enter__()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    pre_events = [(ev(), ev()) for _ in range(args.steps)]
    step_events = [(ev(), ev()) for _ in range(args.steps)]
    launches = 0
    barrier()
    torch.cuda.synchronize(dev)
    clk.mark(0)
    for i in range(args.steps):
        flush.zero_()
        step_events[i][0].record(stream)
        launches += step(pre_events[i])
        step_events[i][1].record(stream)
    torch.cuda.synchronize(dev)
    clk.mark(1)
    clk.__exit__()
    pool.sync()
    barrier()
    step_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in step_events) / args.steps)
    pre_ms = sum(a.elapsed_time(b) for a, b in pre_events) / args.steps
    flops = w.flops()
    value = world * flops / (step_ms / 1e3) / 1e12

    # end to end: pinned host q / new K,V / tables in, attention output out, around the C ABI
    hq = q.cpu().pin_memory()
    hk = kn.cpu().pin_memory()
    hv = vn.cpu().pin_memory()
    hout = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    h2d = hq.numel() * 2 + (hk.numel() + hv.numel()) * 4 + w.tables.nbytes + toks.nbytes + w.slot_mapping.nbytes
    d2h = hout.numel() * 4

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        kn.copy_(hk, non_blocking=True)
        vn.copy_(hv, non_blocking=True)
        step()
        hout.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    # the L2 flush runs between the steps on the same stream: its own device time is taken out
    # of the span (host gaps around it stay in)
    e0, e1 = ev(), ev()
    fl = [(ev(), ev()) for _ in range(args.steps)]
    e0.record(stream)
    for i in range(args.steps):
        fl[i][0].record(stream)
        flush.zero_()
        fl[i][1].record(stream)
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    pool.sync()
    flush_ms = sum(a.elapsed_time(b) for a, b in fl)
    e2e_ms = max_over_ranks((e0.elapsed_time(e1) - flush_ms) / args.steps)
    barrier()
    if rank == 0:
        peak, peak_src = tensor_peak()
        achieved = flops / (pre_ms / 1e3) / 1e12
        line = {
            "metric": PREFILL_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) Q/K/V, seeded block tables)",
            "config": {"workload": describe_prefill(w), "l2": "L2 flushed (256 MiB write) before every step",
                       "parallelism": f"sequence-sharded: {world} GPU(s), one pool each, no collective",
                       "step": "upload tables+slots (1 H2D) + kv_append (16384 tokens) + paged_prefill",
                       "flops_per_step_per_gpu": flops, "queries_per_step_per_gpu": nq},
            "prefill_tokens_per_s": world * nq / (step_ms / 1e3),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic_from_profiles("cfg4"),
                         "kernel": "paged_prefill_tc (tcgen05 QK^T and PV, TMEM accumulators)",
                         "flops_per_launch": flops, "avg_launch_ms": pre_ms, "peak_source": peak_src},
            "e2e": {"value": world * flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                    "path": "pinned host q/K/V/tables in, C-ABI upload + append + prefill, output out",
                    "l2": "the L2 flush between steps is outside the timed span (its device time is subtracted)"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            from oracle import pyoracle as O

            line["cpu_baseline"] = {k: v for k, v in prefill_cpu_baseline(
                w, steps=max(5, args.steps), budget_s=20.0, threads=O.max_threads(), seed=w.seed).items()
                if k != "ms_per_sample"}
        print(json.dumps(line), flush=True)
    pool.close()


BANDWIDTH_CONFIGS = ("append", "append-bf16", "copy", "copy-bf16", "rope-append", "rope-append-bf16")
ROPE_HEADS = 32  # query heads of the rope-append configs (cfg2's Llama-3-8B shape)


def bandwidth_metric(config: str) -> str:
    if config.startswith("rope"):
        return "fused QK-norm + RoPE + KV append"
    return "KV append" if config.startswith("append") else "block copy"


def bandwidth_workload(config: str, rank: int = 0):
    """Seeded inputs of the append / copy configs on the cfg2 arena geometry."""
    nb, hkv, d, bs = 16384, 8, 128, 16
    rng = np.random.default_rng(0x61AC1E5 + 1000003 * rank)
    perm = rng.permutation(nb).astype(np.int32)
    if config.startswith("append") or config.startswith("rope"):
        seqs, chunk = 32, 2048
        tables = perm[: seqs * chunk // bs].reshape(seqs, chunk // bs)
        j = np.arange(chunk)
        slots = (tables[:, j // bs].astype(np.int64) * bs + j % bs).reshape(-1)
        return dict(nb=nb, hkv=hkv, d=d, bs=bs, rng=rng, tables=tables, slots=slots, seqs=seqs, chunk=chunk)
    n_ops = 4096
    return dict(nb=nb, hkv=hkv, d=d, bs=bs, rng=rng, src=perm[:n_ops].copy(), dst=perm[n_ops:2 * n_ops].copy(),
                valid=np.full(n_ops, bs, np.int32))


def bandwidth_cpu_baseline(config: str, steps: int, budget_s: float):
    """The reference's own loops on one host core: the runner's per-token Store loop
    (PagedTransformerRunner.cs:450) or CopyBlockData per fork (PagedBlockPool.cs:304-342), as
    restated in oracle/, on a bounded prefix of the same inputs."""
    from oracle import pyoracle as O

    w = bandwidth_workload(config)
    bf16 = config.endswith("bf16")
    eb = 2 if bf16 else 4
    bs = w["bs"]
    # The sample's blocks are renumbered densely, so the host arena holds only the blocks it
    # touches (the bytes moved are the same; a sparse 2 GiB arena only costs page faults).
    if config.startswith("append") or config.startswith("rope"):
        n = 8192 if config.startswith("append") else 2048
        blk = w["slots"][:n] // bs
        used, inv = np.unique(blk, return_inverse=True)
        slots = (inv.astype(np.int64) * bs + w["slots"][:n] % bs).astype(np.int64)
    else:
        n = 512
        used, inv = np.unique(np.concatenate([w["src"][:n], w["dst"][:n]]), return_inverse=True)
        src, dst = inv[:n].astype(np.int32), inv[n:].astype(np.int32)
    g = O.geom(int(used.size), 1, w["hkv"], w["d"], block_size=bs, dtype=O.BF16 if bf16 else O.F32)
    K, V = O.new_arena(g)
    if config.startswith("rope"):
        k = w["rng"].standard_normal((n, w["hkv"], w["d"]), dtype=np.float32)
        v = w["rng"].standard_normal((n, w["hkv"], w["d"]), dtype=np.float32)
        q = w["rng"].standard_normal((n, ROPE_HEADS, w["d"]), dtype=np.float32)
        pos = (np.arange(n) % 2048).astype(np.int32)
        inv = (500000.0 ** (-2.0 * np.arange(w["d"] // 2) / w["d"])).astype(np.float32)
        qn = np.ones(w["d"], np.float32)
        alg = n * (ROPE_HEADS * w["d"] * 8 + w["hkv"] * 2 * w["d"] * (4 + eb))
        def run():
            O.rope_append(K, V, g, 0, q, k, v, pos, slots, inv, w["d"], 0, 1.0, q_norm=qn, k_norm=qn)
            return 0

        sample = (f"first {n} of the 65536 tokens, per-token bias + QK RMSNorm + RoPE + Store loop, 1 thread "
                  "(the reference's loop is serial)")
    elif config.startswith("append"):
        k = w["rng"].standard_normal((n, w["hkv"], w["d"]), dtype=np.float32)
        v = w["rng"].standard_normal((n, w["hkv"], w["d"]), dtype=np.float32)
        alg = n * w["hkv"] * 2 * w["d"] * (4 + eb)
        run = lambda: O.store_many(K, V, g, 0, slots, k, v)  # noqa: E731
        sample = f"first {n} of the 65536 tokens, per-token Store loop, 1 thread (the reference's loop is serial)"
    else:
        alg = n * w["hkv"] * bs * 2 * w["d"] * eb * 2
        run = lambda: O.copy_many(K, V, g, src, dst, w["valid"][:n])  # noqa: E731
        sample = f"first {n} of the 4096 forks, CopyBlockData per fork, 1 thread (the reference's copy is serial)"
    run()  # touch the pages once
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < steps and time.perf_counter() < t_end:
        t0 = time.perf_counter()
        assert run() == 0
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": alg / med / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": sample + f", median of {len(times)} runs", "ms_per_sample": med * 1e3}


def run_bandwidth(args, world, rank, local, dev, barrier, max_over_ranks):
    """The two data-movement kernels of the pool on their own, each against the HBM roofline, on
    the cfg2 arena geometry (16384 blocks x 8 kv heads x 16 slots x d 128, one layer).

    append: one kv_append of 65536 tokens (32 sequences x 2048 prefill tokens; every sequence's
        slots follow its seeded block table), fp32 sources, fp32 or bf16 arena.
    copy:   one block_copy of 4096 full blocks (seeded distinct src / dst), K and V.
    Both move about 1 GB per launch, more than L2.  Weak scaling: every rank owns a pool."""
    import torch

    import glacier_kv as G

    dtype = "bf16" if args.config.endswith("bf16") else "f32"
    eb = 2 if dtype == "bf16" else 4
    w = bandwidth_workload(args.config, rank)
    nb, hkv, d, bs, rng = w["nb"], w["hkv"], w["d"], w["bs"], w["rng"]
    pool = G.PagedBlockPool(nb, 1, hkv, d, bs, d, device=local, dtype=dtype)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    if args.config.startswith("rope"):
        seqs, chunk, tables, slots = w["seqs"], w["chunk"], w["tables"], w["slots"]
        n_tok = slots.size
        pool.reserve_step(seqs, tables.shape[1], n_tok, ROPE_HEADS)
        pool.upload_step(tables, np.full(seqs, chunk, np.int32), slots, stream=stream)
        kn = torch.from_numpy(rng.standard_normal((n_tok, hkv, d), dtype=np.float32)).to(dev)
        vn = torch.from_numpy(rng.standard_normal((n_tok, hkv, d), dtype=np.float32)).to(dev)
        q0 = torch.from_numpy(rng.standard_normal((n_tok, ROPE_HEADS, d), dtype=np.float32)).to(dev)
        qn = torch.ones(d, device=dev)
        pos = (np.arange(n_tok) % chunk).astype(np.int32)
        # q read + written, k and v read as fp32 and written in the arena's type
        alg = n_tok * (ROPE_HEADS * d * 8 + hkv * 2 * d * (4 + eb))

        def launch():
            pool.rope_append(0, q0, kn, vn, pos, ROPE_HEADS, freq_base=500000.0, q_norm=qn, k_norm=qn,
                             stream=stream)
            return pool.last_launch_count

        hq, hk, hv = q0.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory()
        h2d, d2h = (hq.numel() + hk.numel() + hv.numel()) * 4, hq.numel() * 4
        hq_out = torch.empty_like(hq).pin_memory()

        def e2e():
            q0.copy_(hq, non_blocking=True)
            kn.copy_(hk, non_blocking=True)
            vn.copy_(hv, non_blocking=True)
            launch()
            hq_out.copy_(q0, non_blocking=True)

        kernel = (f"rope_append_kernel<{'bf16' if eb == 2 else 'float'}, 4> ({n_tok} tokens: {ROPE_HEADS} q rows "
                  f"in place, {hkv} k and v rows into the arena)")
        work = (f"{args.config}: bias-free QK RMSNorm + NEOX RoPE (base 5e5) of {n_tok} tokens ({seqs} seqs x "
                f"{chunk}), {ROPE_HEADS}q/{hkv}kv heads, d {d}, fp32 q/k/v, {dtype} arena, block {bs}, pool {nb} blocks")
    elif args.config.startswith("append"):
        seqs, chunk, tables, slots = w["seqs"], w["chunk"], w["tables"], w["slots"]
        n_tok = slots.size
        pool.reserve_step(seqs, tables.shape[1], n_tok, hkv)
        pool.upload_step(tables, np.full(seqs, chunk, np.int32), slots, stream=stream)
        kn = torch.from_numpy(rng.standard_normal((n_tok, hkv, d), dtype=np.float32)).to(dev)
        vn = torch.from_numpy(rng.standard_normal((n_tok, hkv, d), dtype=np.float32)).to(dev)
        alg = n_tok * hkv * 2 * d * (4 + eb)  # fp32 rows read, arena rows written

        def launch():
            pool.kv_append(0, kn, vn, stream=stream)
            return pool.last_launch_count

        hk, hv = kn.cpu().pin_memory(), vn.cpu().pin_memory()
        h2d, d2h = hk.numel() * 4 * 2, 0

        def e2e():
            kn.copy_(hk, non_blocking=True)
            vn.copy_(hv, non_blocking=True)
            launch()

        kernel = f"kv_append_kernel<{'bf16' if eb == 2 else 'float'}> (65536 tokens x 8 heads, K and V rows)"
        work = (f"{args.config}: kv_append of {n_tok} tokens ({seqs} seqs x {chunk}), {hkv} kv heads, d {d}, "
                f"fp32 sources, {dtype} arena, block {bs}, pool {nb} blocks")
    else:
        src, dst, valid = w["src"], w["dst"], w["valid"]
        n_ops = src.size
        alg = n_ops * hkv * bs * 2 * d * eb * 2  # K and V spans, read + written

        def launch():
            pool.block_copy(src, dst, valid, stream=stream)
            return pool.last_launch_count

        h2d, d2h = n_ops * 3 * 4, 0
        e2e = launch
        kernel = f"block_copy_kernel ({n_ops} full blocks, K and V)"
        work = (f"{args.config}: block_copy of {n_ops} full blocks (seeded distinct src/dst), {hkv} kv heads, "
                f"d {d}, {dtype} arena, block {bs}, pool {nb} blocks")

    clk = Clocks(dev)
    clk.__enter__()
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize(dev)
    events = [(ev(), ev()) for _ in range(args.steps)]
    launches = 0
    barrier()
    torch.cuda.synchronize(dev)
    clk.mark(0)
    for i in range(args.steps):
        events[i][0].record(stream)
        launches += launch()
        events[i][1].record(stream)
    torch.cuda.synchronize(dev)
    clk.mark(1)
    clk.__exit__()
    pool.sync()
    barrier()
    ms_local = sum(a.elapsed_time(b) for a, b in events) / args.steps
    ms = max_over_ranks(ms_local)
    for _ in range(args.warmup):
        e2e()
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = ev(), ev()
    e0.record(stream)
    for _ in range(args.steps):
        e2e()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    pool.sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    barrier()
    if rank == 0:
        peak, peak_kind = peaks()
        achieved = alg / (ms_local / 1e3) / 1e9
        line = {
            "metric": f"{bandwidth_metric(args.config)} GB/s per B200 vs HBM peak",
            "value": world * alg / (ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded N(0,1) rows, seeded block tables)",
            "config": {"workload": work, "l2": f"inputs larger than L2 ({alg / 1e9:.2f} GB moved per launch)",
                       "parallelism": f"{world} GPU(s), one pool each, no collective",
                       "bytes_per_step_per_gpu": alg},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic_from_profiles(args.config),
                         "kernel": kernel, "bytes_per_launch": alg, "avg_launch_ms": ms_local,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s"},
            "e2e": {"value": world * alg / (e2e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                    "path": ("pinned host q/K/V rows copied in, gkv_rope_append, rotated q copied out"
                             if args.config.startswith("rope") else
                             "pinned host K/V rows copied in, then gkv_kv_append" if args.config.startswith("append")
                             else "gkv_block_copy from host op lists (ops copied in by the call)")},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = {k: v for k, v in bandwidth_cpu_baseline(
                args.config, steps=max(5, args.steps), budget_s=20.0).items() if k != "ms_per_sample"}
        print(json.dumps(line), flush=True)
    pool.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg3")
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="sequences of cfg2/cfg3 (default: the config's own); for small profiler captures")
    ap.add_argument("--share", type=int, default=0,
                    help="cfg3 / cfg5 on one GPU: decode only rank 0's share of an N-GPU split (cfg3: its "
                         "longest-first sequences; cfg5: its block range, without the exchange) -- the per-rank "
                         "step of the N-GPU run, for profiling it on one GPU")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import glacier_kv as G
    from glacier_kv import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.config == "cfg4" or args.config in BANDWIDTH_CONFIGS:
        run = run_prefill if args.config == "cfg4" else run_bandwidth
        run(args, world, rank, local, dev, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        return

    w = workload(args.config, rank, world, args.batch)
    global_batch = (args.batch or 256) if args.config in CFG3 else w.batch
    if args.share > 1 and world == 1 and args.config in CFG3:
        from glacier_kv import workloads as W

        w = W.lpt_share(w, 0, args.share)
        global_batch = w.batch  # this GPU decodes its share only
    elif args.share > 1 and world == 1 and args.config == "cfg5":
        from glacier_kv import workloads as W

        w = W.cfg5_local(0, args.share, W.SEED)  # rank 0's block range, decoded without the exchange
        global_batch = w.batch
    pool = W.make_pool(w, device=local)
    W.fill_arena_randn(pool, seed=w.seed)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(w.seed + 17)
    q = torch.from_numpy(rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)).to(dev)
    n_tok = int(w.slot_mapping.size)
    kn = torch.from_numpy(rng.standard_normal((max(n_tok, 1), w.heads_kv, w.head_dim)).astype(np.float32)).to(dev)
    vn = torch.from_numpy(rng.standard_normal((max(n_tok, 1), w.heads_kv, w.v_head_dim)).astype(np.float32)).to(dev)
    out = torch.zeros((w.batch, w.n_heads, w.v_head_dim), dtype=torch.float32, device=dev)
    max_blocks = w.tables.shape[1]
    pool.reserve_step(w.batch, max_blocks, max(n_tok, 1), w.n_heads)
    kv_bytes = w.kv_bytes()
    small = kv_bytes < 2 * 126e6  # working set within reach of L2: flush between steps
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if small else None

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    # long-context split-KV (cfg5) over several GPUs: each rank holds its block range and the
    # step ends with the NCCL exchange + LSE merge; total work is fixed (strong scaling)
    split_kv = args.config == "cfg5" and world > 1
    comm = None
    if split_kv:
        uid = [G.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = G.Comm(uid[0], world, rank, local, timeout_ms=120_000)

    def decode():
        if split_kv:
            pool.paged_decode_splitkv_dist(comm, 0, q, out, w.n_heads, w.scale, stream=stream)
        else:
            pool.paged_decode(0, q, out, w.n_heads, w.scale, stream=stream)

    def step(timed_decode=None):
        pool.upload_step(w.tables, w.ctx_lens, w.slot_mapping, stream=stream)
        launches = 0
        if n_tok:
            pool.kv_append(0, kn[:n_tok], vn[:n_tok], stream=stream)
            launches += pool.last_launch_count
        if timed_decode is not None:
            timed_decode[0].record(stream)
        decode()
        if timed_decode is not None:
            timed_decode[1].record(stream)
        return launches + pool.last_launch_count

    clk = Clocks(dev)
    clk.__enter__()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # ---- device-resident timing ----
    # Inputs larger than L2: the K steps run back to back and are timed as one span (events
    # only at its ends, so nothing comes between consecutive steps' launches).  Smaller
    # working sets: an L2 flush between steps, each step timed by its own events.  The decode
    # launches' own duration (the roofline's denominator) is timed in a second loop.
    dec_events = [(ev(), ev()) for _ in range(args.steps)]
    step_events = [(ev(), ev()) for _ in range(args.steps)]
    launches = 0
    barrier()
    torch.cuda.synchronize(dev)
    clk.mark(0)
    t0 = ev()
    t0.record(stream)
    h0 = time.perf_counter()
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
            step_events[i][0].record(stream)
            launches += step(dec_events[i])
            step_events[i][1].record(stream)
        else:
            launches += step()
    t1 = ev()
    t1.record(stream)
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # enqueue cost per step on the host
    torch.cuda.synchronize(dev)
    clk.mark(1)
    clk.__exit__()
    barrier()
    torch.cuda.synchronize(dev)
    span_ms = t0.elapsed_time(t1) / args.steps
    if flush is not None:
        step_ms = sum(a.elapsed_time(b) for a, b in step_events) / args.steps
    else:
        for i in range(args.steps):  # the decode launches alone, for the roofline
            step(dec_events[i])
        torch.cuda.synchronize(dev)
        step_ms = span_ms
    ms = max_over_ranks(step_ms)
    dec_ms = sum(a.elapsed_time(b) for a, b in dec_events) / args.steps
    breakdown = None
    if split_kv:
        # the same decode of this rank's block ranges without the exchange: what the exchange and
        # the cross-rank merge add to a split-KV decode
        lse = torch.empty((w.batch, w.n_heads), dtype=torch.float32, device=dev)
        tmp = torch.empty_like(out)
        loc = [(ev(), ev()) for _ in range(args.steps)]
        for i in range(args.steps):
            pool.upload_step(w.tables, w.ctx_lens, w.slot_mapping, stream=stream)
            loc[i][0].record(stream)
            pool.paged_decode_lse(0, q, tmp, lse, w.n_heads, w.scale, stream=stream)
            loc[i][1].record(stream)
        torch.cuda.synchronize(dev)
        local_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in loc) / args.steps)
        dist_ms = max_over_ranks(dec_ms)
        breakdown = {"local_decode_ms": local_ms, "split_kv_call_ms": dist_ms,
                     "exchange_and_merge_ms": dist_ms - local_ms,
                     "what": "max over ranks of: this rank's decode with lse alone, and the whole "
                             "gkv_paged_decode_splitkv_dist call (decode + peer push + bounded wait + LSE merge)"}
    # strong-scaled configs split one global batch over the ranks; the others add a batch per rank
    seqs_per_step = global_batch if args.config in STRONG else world * w.batch
    value = seqs_per_step / (ms / 1e3)

    # ---- end-to-end through the C ABI with host buffers ----
    hq = q.cpu().pin_memory()
    hk = kn[:max(n_tok, 1)].cpu().pin_memory()
    hv = vn[:max(n_tok, 1)].cpu().pin_memory()
    hout = torch.empty((w.batch, w.n_heads, w.v_head_dim), dtype=torch.float32).pin_memory()
    meta_bytes = w.tables.nbytes + w.ctx_lens.nbytes + w.slot_mapping.nbytes
    h2d = hq.numel() * 4 + (hk.numel() + hv.numel()) * 4 * (1 if n_tok else 0) + meta_bytes
    d2h = hout.numel() * 4

    def e2e_step():
        if split_kv:  # host q in, host output out, around the distributed C-ABI call
            q.copy_(hq, non_blocking=True)
            pool.upload_step(w.tables, w.ctx_lens, w.slot_mapping, stream=stream)
            decode()
            hout.copy_(out, non_blocking=True)
        else:
            pool.decode_step_host(0, w.tables, w.ctx_lens, w.slot_mapping, hk, hv, hq, hout, w.n_heads, w.scale,
                                  stream=stream)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    # the L2 flush (small working sets) runs between the steps on the same stream: its own
    # device time is taken out of the span (host gaps around it stay in)
    e0, e1 = ev(), ev()
    fl = [(ev(), ev()) for _ in range(args.steps)] if flush is not None else []
    e0.record(stream)
    for i in range(args.steps):
        if flush is not None:
            fl[i][0].record(stream)
            flush.zero_()
            fl[i][1].record(stream)
        e2e_step()
    if not split_kv:  # the last call's output copy runs on the pool's copy stream
        pool.wait_host_outputs(stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    flush_ms = sum(a.elapsed_time(b) for a, b in fl)
    e2e_ms = max_over_ranks((e0.elapsed_time(e1) - flush_ms) / args.steps)
    barrier()

    if rank == 0:
        peak, peak_kind = peaks()
        alg_bytes = kv_bytes + w.qo_bytes()
        achieved = alg_bytes / (dec_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.config in STRONG else "weak",
            "vs_baseline": None, "dtype": "f32", "kv_dtype": w.dtype,
            "data": "synthetic (seeded N(0,1) Q/K/V, seeded block tables)",
            "config": {"workload": describe(w),
                       "l2": "L2 flushed (256 MiB write) before every step" if small else
                             f"inputs larger than L2 ({kv_bytes / 1e9:.2f} GB of KV read per step)",
                       "parallelism": (f"split-KV: each sequence's blocks split over {world} GPU(s), (out, lse) "
                                       "exchanged through peer-memory mailboxes (NCCL all-gather fallback) + LSE "
                                       "merge") if split_kv else
                                      (f"rank 0's block range of each sequence split over {args.share} GPUs, decoded "
                                       "alone on one GPU without the exchange")
                                      if args.share > 1 and args.config == "cfg5" else
                                      (f"rank 0's share ({w.batch} sequences) of the 256 split over {args.share} GPUs "
                                       "by longest-first partitioning, run alone on one GPU")
                                      if args.share > 1 else
                                      (f"sequence-sharded: the {global_batch} sequences split over {world} GPU(s) by "
                                       "longest-first partitioning, one pool each, no collective")
                                      if args.config in STRONG else
                                      f"sequence-sharded: {world} GPU(s), one pool each, no collective",
                       "step": ("upload tables (1 H2D) + split-KV decode with lse + peer exchange + LSE merge"
                                if split_kv else
                                "upload tables+slots (1 H2D) + kv_append + paged_decode (+ merge kernel)"
                                if n_tok else "upload tables (1 H2D) + paged_decode (+ merge kernel)")},
            "kv_gbs_per_gpu": kv_bytes / (ms / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic_from_profiles(args.config),
                         "kernel": "paged_decode (split-KV decode kernel; merge fused or a second launch for long splits)",
                         "bytes_per_launch": alg_bytes, "avg_launch_ms": dec_ms,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s"},
            "e2e": {"value": seqs_per_step / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                    "path": ("pinned host q copied in, gkv_upload_step + gkv_paged_decode_splitkv_dist, "
                             "output copied out (both copies on the step's stream)") if split_kv else
                            "gkv_decode_step_host (pinned host q/K/V/tables in, output out)",
                    "l2": ("the L2 flush between steps is outside the timed span (its device time is "
                           "subtracted)") if flush is not None else "no flush (inputs larger than L2)"},
            "gpu_launches": launches,
            "host_enqueue_ms_per_step": host_ms,
            "clocks": clk.summary(),
        }
        if breakdown is not None:
            line["split_kv_breakdown"] = breakdown
        if not args.no_cpu_baseline and world == 1:
            from oracle import pyoracle as O

            line["cpu_baseline"] = {k: v for k, v in cpu_baseline_run(
                w, steps=max(5, args.steps), budget_s=20.0, threads=O.max_threads(), seed=w.seed).items()
                if k != "ms_per_sample"}
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    pool.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
