#!/usr/bin/env python
"""Benchmark of the Fathom key-scan decode step on B200.

Headline workload: Qwen3-8B attention shape (8 KV heads, G=4, D=128),
batch 1, T = 1,048,576 tokens, 36 layers, budget 48 (the paper's 56-bit "Fathom 48"),
k = 512 + 4 sink + 64 local.  The bit-plane index (copy-index order) and the bf16 K/V rows live
in pinned, mapped host memory.  One step = one decode step = for each of the 36 layers:
plan -> zero-copy plane-prefix scan of the host index -> sink+local top-k -> unique-row
zero-copy gather + exact attention.  Layers run back to back on one stream (a layer's query
depends on the previous layer's output in a real model).

  value   scanned key-rows/s = T * Hkv * layers / step time, inputs (q, g) already on the device
  e2e     the same through the public API with host buffers: every step copies that step's
          queries and gains from pinned host memory and reads the attention outputs back
  roofline  the scan kernel: algorithmic bytes (bytes_planes of each layer's plan) / its mean
          CUDA-event duration (events recorded on the launching stream right before the scan call and,
          by the library, right after the scan kernel), against the host link bandwidth measured in
          this run (pinned H2D cudaMemcpy, 1 GiB)
  hbm_resident  config 1 (T = 131072, index + K/V in HBM) as a secondary figure, against
          MEASURED_PEAKS.json hbm_gbs (with the Chan4 comparator scans and the KLT-store step)
  chan4_host  the reference's channel-subset comparators (SparQ r = 16, 32 channels) on the same
          host-resident step, for the head-to-head of its offload table
  copy_index_host  the same step through the reference's copy-index index path (the planes a layer
          needs staged into device memory in 1, 4 or 8 pipelined chunks, each scanned from HBM)
  hf_decode  end to end through a Qwen3-8B-shaped transformers model (random weights) whose attention
          is patched onto this path, synthetic KV cache in host memory at 256k and 1M tokens: wall and
          CUDA-graph device ms per generated token (`--part hf` adds 512k)
  cpu_baseline  the CPU oracle (numpy restatement of the reference path) on a bounded sample

`--impl reference` times the reference's CPU path (the oracle port; the reference is Python and
its checkout is not on the GPU box) on bounded samples of the same workload.
Multi-GPU (torchrun, N > 1): the context is split into contiguous 64-token-aligned chunks of T
tokens per rank (weak scaling: N*T total); each rank scans its chunk, keeps its local top-k, and
an NCCL all-gather plus a merge produce the global top-k; attention partials are combined the
same way.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["fathom", "reference"], default="fathom")
    ap.add_argument("--ctx", type=int, default=1048576, help="tokens per rank")
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--kv-buffers", type=int, default=4, help="distinct host K/V row buffers, cycled over layers")
    ap.add_argument("--kv-layout", choices=["interleaved", "separate"], default="interleaved",
                    help="host K/V rows: one [BH][T][2][128] cache (K and V of a token adjacent) or two buffers")
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--g", type=int, default=4)
    ap.add_argument("--budget", type=float, default=48.0)
    ap.add_argument("--k", type=int, default=512)
    ap.add_argument("--sink", type=int, default=4)
    ap.add_argument("--local", type=int, default=64)
    ap.add_argument("--hbm-ctx", type=int, default=131072)
    ap.add_argument("--no-hbm", action="store_true", help="skip the HBM-resident secondary figure")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-hf", action="store_true", help="skip the end-to-end transformers-model figure")
    ap.add_argument("--hf-ctx", default="", help="--part hf: comma-separated context lengths (default 256k, 512k, 1M)")
    ap.add_argument("--cpu-heads", type=int, default=2, help="KV heads of one layer in the CPU sample")
    ap.add_argument("--part", choices=["all", "host", "hbm", "config3", "hf", "scan"], default="all",
                    help="profiling runs: only the host-resident step (host), only the HBM-resident figure (hbm), "
                         "or scan launches alone over --scan-layers layers of --scan-spec (scan)")
    ap.add_argument("--scan-spec", choices=["config1", "config3"], default="config1")
    ap.add_argument("--scan-layers", type=int, default=36, help="--part scan: layers whose rows one launch covers")
    return ap.parse_args()


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ clocks
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix=f"fathom_clocks_{self.index}_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception as e:  # nvidia-smi missing: report no clocks
            log("clock sampling unavailable:", e)
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------------ helpers
def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class LinkProbe:
    """One round of the host-link roofline: a pinned host -> device cudaMemcpy of 1 GiB (DMA engine).
    Returns (bytes, seconds) by CUDA events."""

    def __init__(self, dev):
        self.n = 1 << 30
        self.h = torch.empty(self.n, dtype=torch.uint8, pin_memory=True)
        self.d = torch.empty(self.n, dtype=torch.uint8, device=dev)

    def __call__(self):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.d.copy_(self.h, non_blocking=True)
        e1.record()
        e1.synchronize()
        return self.n, e0.elapsed_time(e1) * 1e-3

    def free(self):
        del self.h, self.d


class SMReadProbe:
    """One round of the ceiling of SM-issued reads of pinned mapped host memory (the scan's kind of
    reads): a plain vectorised element-wise kernel (torch int32 add) reading a 1 GiB mapped alias and
    writing HBM.  Zero-copy reads are capped here, below the DMA copy.  Returns (bytes, seconds)."""

    def __init__(self, dev, off):
        self.n = 1 << 28
        self.buf = off.MappedBuffer((self.n,), torch.int32, dev)
        self.buf.host.zero_()
        self.d = torch.empty(self.n, dtype=torch.int32, device=dev)

    def __call__(self):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.add(self.buf.dev, 0, out=self.d)
        e1.record()
        e1.synchronize()
        return self.n * 4, e0.elapsed_time(e1) * 1e-3

    def free(self):
        del self.d
        self.buf.free()


def probe_gbs(probe, world):
    """(aggregate GB/s, per-rank GB/s): best of 6 alone at N = 1; at N > 1 every rank runs the probe at
    the same time (barrier-synchronised rounds), the aggregate being all bytes over the slowest rank."""
    try:
        if world == 1:
            best = max(b / s for b, s in (probe() for _ in range(6))) / 1e9
            return best, [best]
        from fathom_b200 import shard
        agg, per = shard.concurrent_probe(probe, rounds=5, sync=torch.cuda.synchronize)
        return agg / 1e9, [v / 1e9 for v in per]
    finally:
        probe.free()


class Layer:
    pass


def host_budget(a):
    """How many distinct index layers and K/V row buffers this rank can pin: everything the local ranks
    pin must stay under 75% of the host's available memory (the rest is cycled over the layers)."""
    avail = 0
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    nblk = -(-a.ctx // 64)
    per_index = a.hkv * 128 * nblk * (4 * 8 + 2)          # planes + scales of one layer
    per_kv = 2 * a.hkv * a.ctx * 128 * 2                   # K and V rows of one layer
    budget = 0.75 * avail / local if avail else float("inf")
    n_kv = max(1, min(a.kv_buffers, a.layers))
    n_index = a.layers
    while n_index * per_index + n_kv * per_kv > budget and n_kv > 1:
        n_kv -= 1
    while n_index * per_index + n_kv * per_kv > budget and n_index > 1:
        n_index -= 1
    return n_index, n_kv


def build_host_layers(a, dev, rank, world, bp, off):
    """Per layer: a host-order store of this rank's context chunk in mapped host memory, the layer's
    query and gain on the device; K/V row buffers for the first kv_buffers layers.  If the host cannot
    pin a distinct index for every layer, later layers reuse the first indexes (same bytes moved)."""
    layers, kv = [], []
    BH = a.hkv
    n_index, a.kv_buffers = host_budget(a)
    a.index_buffers = n_index
    for L in range(a.layers):
        if L >= n_index:                     # host memory exhausted: reuse an index (queries still differ)
            src = layers[L % n_index]
            lay = Layer()
            qgen = torch.Generator(device=dev).manual_seed(777 + L)
            scale = torch.randn(BH, 1, 128, generator=qgen, device=dev).exp()
            lay.q = (torch.randn(BH, a.g, 128, generator=qgen, device=dev) * scale).contiguous()
            lay.g = ((lay.q ** 2) * (scale[:, 0, None, :] ** 2)).sum(1).contiguous()
            lay.store = src.store
            plan = bp.make_plan(lay.g, a.budget)
            lay.bytes = bp.bytes_planes(plan["t"], a.ctx)
            layers.append(lay)
            continue
        gen = torch.Generator(device=dev).manual_seed(1000 * (rank + 1) + L)
        qgen = torch.Generator(device=dev).manual_seed(777 + L)     # same query on every rank
        scale = torch.randn(BH, 1, 128, generator=qgen, device=dev).exp()
        q = torch.randn(BH, a.g, 128, generator=qgen, device=dev) * scale
        K = (torch.randn(BH, a.ctx, 128, generator=gen, device=dev) * scale).to(torch.bfloat16)
        lay = Layer()
        lay.q = q.contiguous()
        lay.g = ((q ** 2) * (scale[:, 0, None, :] ** 2)).sum(1).contiguous()   # Var(K) = scale^2 (same on all ranks)
        lay.store = off.HostPlaneStore(K)
        plan = bp.make_plan(lay.g, a.budget)
        lay.bytes = bp.bytes_planes(plan["t"], a.ctx)
        lay.nact = float(plan["nact"].float().mean())
        if L < a.kv_buffers:
            V = (torch.randn(BH, a.ctx, 128, generator=gen, device=dev) * scale).to(torch.bfloat16)
            if a.kv_layout == "interleaved":
                buf = off.MappedBuffer((BH, a.ctx, 2, 128), torch.bfloat16, dev)
                buf.dev[:, :, 0].copy_(K)
                buf.dev[:, :, 1].copy_(V)
                kv.append({"K": buf.dev[:, :, 0], "V": buf.dev[:, :, 1], "bufs": [buf]})
            else:
                kb = off.MappedBuffer(K.shape, torch.bfloat16, dev)
                vb = off.MappedBuffer(V.shape, torch.bfloat16, dev)
                kb.dev.copy_(K)
                vb.dev.copy_(V)
                kv.append({"K": kb.dev, "V": vb.dev, "bufs": [kb, vb]})
            del V
        del K
        torch.cuda.synchronize(dev)
        layers.append(lay)
    return layers, kv


def decode_step_1gpu(a, layers, kv, bp, off, scores, outs, q_in=None, g_in=None, scan_events=None):
    """One decode step over all layers (device-resident q/g unless q_in/g_in given)."""
    k_tot = a.k + a.sink + a.local
    for L, lay in enumerate(layers):
        q = lay.q if q_in is None else q_in[L]
        g = lay.g if g_in is None else g_in[L]
        plan = bp.make_plan(g, a.budget)
        if scan_events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e1.record()    # creates the handle; the library records it again right after the scan kernel
            e0.record()
        idx = bp.scan_topk(lay.store, q, plan, k_tot, a.sink, a.local, scores=scores,
                           scan_done_event=e1 if scan_events is not None else None)
        if scan_events is not None:
            scan_events.append((e0, e1, lay.bytes))
        rows = kv[L % len(kv)]
        outs[L] = off.decode_attention(q, idx, rows["K"], rows["V"], a.ctx)
    return outs


# ------------------------------------------------------------------ CPU baseline (oracle port)
def cpu_sample(a, heads, seed_layer=0):
    """The reference path on the host cores (numpy oracle, all BLAS threads): plan + scan +
    sink_local_topk + gather/attention for `heads` KV heads of one layer at T = a.ctx.
    Returns (seconds, key-rows)."""
    from oracle import bitplane_oracle as O
    g = torch.Generator().manual_seed(4242 + seed_layer)
    scale = torch.randn(heads, 1, 128, generator=g).exp()
    K = (torch.randn(heads, a.ctx, 128, generator=g) * scale).to(torch.bfloat16).float().numpy()
    V = (torch.randn(heads, a.ctx, 128, generator=g) * scale).to(torch.bfloat16).float().numpy()
    q = (torch.randn(heads, a.g, 128, generator=g) * scale).numpy()
    gain = ((q ** 2) * (scale[:, 0].numpy() ** 2)[:, None, :]).sum(1)
    code, sc = O.quantise_u4(K)               # offline store build: not timed
    k_tot = a.k + a.sink + a.local
    t0 = time.perf_counter()
    plan = O.make_plan(gain, a.budget)
    s = O.scan_scores_threaded(q, code, sc, plan["t"], os.cpu_count())
    idx = O.sink_local_topk(s, k_tot, a.sink, a.local)
    O.decode_attention(q, K, V, idx)
    return time.perf_counter() - t0, heads * a.ctx


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(a, rank, world):
    """--impl reference: rank 0 times the CPU reference path (oracle port) per step on a bounded
    sample; other ranks exit without work."""
    if rank != 0:
        return
    cores = os.cpu_count()
    for _ in range(a.warmup):
        cpu_sample(a, 1)
    ts, rows = [], 0
    for s in range(a.steps):
        t, r = cpu_sample(a, 1, seed_layer=s)
        ts.append(t)
        rows = r
    tmean = float(np.mean(ts))
    val = rows / tmean
    sample = (f"1 KV head x {a.ctx} tokens of one layer per step (plan+scan+sink_local_topk+attention), "
              f"numpy oracle restatement with the scan on a {cores}-thread pool, {cpu_model()}; scaled to key-rows/s")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "key-rows/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": tmean * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(a, world),
            "cpu_baseline": {"value": val, "unit": "key-rows/s", "cores": cores, "kind": "port", "sample": sample,
                             "cpu_model": cpu_model()},
            "e2e": {"value": val, "unit": "key-rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


METRIC = "scanned key-rows/s and decode-step us at 1M ctx, 56-bit, k=512 (1/2/4/8 GPU)"

# Per-launch traffic of the scan kernel relative to its algorithmic bytes, from one ncu capture each
# (small cases of the same kernels; the ratio is size-independent because every launch reads each
# needed plane run once):
#   host run order, zero-copy: pcie__read_bytes.sum = 15,359,488 B for 14,151,680 algorithmic bytes
#     (T = 262144, 8 KV heads, budget 48, bulk-copy instance)
#   HBM order, phase kernel: dram__bytes_read.sum = 312,030,464 B for 254,251,008 algorithmic bytes (36
#     layers x 8 KV heads of T = 131072, budget 48, one launch); a single layer's 16.8 MB of scores stay in
#     L2 between the scan and the selection (dram__bytes_write.sum 0 in a per-layer capture of the
#     bulk-copy kernel, same shape), so the per-layer figure counts reads only
TRAFFIC_RATIO_HOST = 15359488 / 14151680
TRAFFIC_RATIO_HBM = 312030464 / 254251008
# config 3, one layer's fused scan launch (group keys; scores kept in L2 by an evict-last policy):
# ncu dram__bytes_read.sum 35,097,856 B + dram__bytes_write.sum 43,120,640 B (the fp32 scores of
# 32 rows x 7 heads x 131072 tokens that leave L2) over 28,274,688 algorithmic index bytes
TRAFFIC_RATIO_HBM3 = (35097856 + 43120640) / 28274688


def config_dict(a, world):
    return {"workload": "config2: host-resident index + K/V rows, Qwen3-8B attention shape, decode step",
            "ctx_per_gpu": a.ctx, "ctx_total": a.ctx * world, "layers": a.layers, "kv_heads": a.hkv,
            "q_per_kv": a.g, "head_dim": 128, "batch": 1, "budget": a.budget, "k": a.k, "sink": a.sink,
            "local": a.local, "kv_row_buffers": a.kv_buffers, "kv_layout": a.kv_layout,
            "index_buffers": getattr(a, "index_buffers", a.layers),
            "parallelism": "context-shard" + str(world) if world > 1 else "single",
            "l2": "inputs larger than L2 (host index per step >> 126 MB)"}


# ------------------------------------------------------------------ HBM-resident secondary figure
HBM_SPECS = {
    "config1": dict(hkv=8, g=4, n=131072, layers=36, k=512, batch=1,
                    workload="config1: HBM-resident index + K/V, Qwen3-8B shape, T=131072, 36 layers, graph-captured step"),
    "config3": dict(hkv=4, g=7, n=131072, layers=28, k=2048, batch=8,
                    workload="config3: HBM-resident, Qwen2.5-7B shape (4 KV heads, G=7), 8 sequences x T=131072, "
                             "28 layers, k=2048+4+64, graph-captured step"),
}


def hbm_figure(a, dev, bp, off, peaks, spec="config1", batch=None, seed=None):
    """A decode step with index and K/V rows in HBM (one CUDA graph per step), and the scan kernel's
    mean duration from a graph of back-to-back scans."""
    from fathom_b200.synth import make_layer
    sp = HBM_SPECS[spec]
    n, BH, G, nl = sp["n"], sp["hkv"] * (batch or sp["batch"]), sp["g"], sp["layers"]
    if spec == "config1":
        n = a.hbm_ctx
    layers, kvs = [], []
    for L in range(nl):
        d = make_layer(BH, G, n, seed=seed if seed is not None else (1 if spec == "config1" else 3), layer=L, device=dev, kv_dtype=torch.bfloat16,
                       with_v=True)
        lay = Layer()
        lay.store = bp.PlaneStore(d["K"])
        lay.store_K = d["K"] if (spec == "config1" and L < 4) else None
        lay.q, lay.g = d["q"], d["g"]
        lay.bytes = bp.bytes_planes(bp.make_plan(d["g"], a.budget)["t"], n)
        kvs.append((d["K"], d["V"]))
        layers.append(lay)
        del d
    k_tot = sp["k"] + a.sink + a.local
    scores = torch.empty(BH, G, n, device=dev)

    def step(budget):
        for L, lay in enumerate(layers):
            plan = bp.make_plan(lay.g, budget)
            idx = bp.scan_topk(lay.store, lay.q, plan, k_tot, a.sink, a.local, scores=scores)
            off.decode_attention(lay.q, idx, kvs[L][0], kvs[L][1], n)

    def timed_step(budget, profile=False):
        for _ in range(a.warmup):
            step(budget)
        torch.cuda.synchronize()
        # graph of the whole step removes the per-launch host cost from the per-layer latency
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(budget)
        torch.cuda.synchronize()
        for _ in range(a.warmup):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if profile:
            torch.cuda.profiler.start()
        e0.record()
        for _ in range(a.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        if profile:
            torch.cuda.profiler.stop()
        del g
        return e0.elapsed_time(e1) / a.steps

    ms = timed_step(a.budget, profile=True)
    sweep = []
    if spec == "config1":
        # the other budgets of the configuration (about 47 and 92 bits per row on real keys)
        for b in (40.0, 80.0):
            bits = float(np.mean([bp.bytes_planes(bp.make_plan(lay.g, b)["t"], n) for lay in layers])) * 8 / (n * BH)
            sweep.append({"budget": b, "bits_per_row": bits, "ms_per_step": timed_step(b)})
    # the scan kernel alone, back to back in a graph (launch gaps removed): mean duration per layer
    plans = [bp.make_plan(lay.g, a.budget) for lay in layers]
    gs = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gs):
        for lay, plan in zip(layers, plans):
            lay.store.scan(lay.q, plan, out=scores)
    for _ in range(3):
        gs.replay()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(a.steps):
        gs.replay()
    f1.record()
    torch.cuda.synchronize()
    scan_ms = f0.elapsed_time(f1) / (a.steps * len(layers))
    del gs
    batched = batched_scan_figure(a, bp, layers, n, BH, G, peaks)
    byts = [lay.bytes for lay in layers]
    comparators = chan4_figure(a, bp, layers, peaks, n, BH, scores) if spec == "config1" else None
    klt_step = klt_figure(a, bp, off, layers, kvs, n, BH, k_tot, scores) if spec == "config1" else None
    achieved = float(np.mean(byts)) / (scan_ms * 1e-3) / 1e9
    rows = n * BH * nl
    del layers, kvs
    torch.cuda.empty_cache()
    return {"workload": sp["workload"],
            "value": rows / (ms * 1e-3), "unit": "key-rows/s", "ms_per_step": ms,
            "scan_ms_per_layer": scan_ms, "scan_timing": f"{nl} scan launches in one CUDA graph, mean per launch",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"],
                         "traffic": float(np.mean(byts)) * (TRAFFIC_RATIO_HBM if spec == "config1"
                                                            else TRAFFIC_RATIO_HBM3),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch (same shape)"
                                           + ("" if spec == "config1" else
                                              "; writes are the fp32 scores that leave L2 (the selection reads "
                                              "them back), reads 1.23x the algorithmic bytes"),
                         "bytes_per_launch": float(np.mean(byts))},
            "bits_per_row": float(np.mean(byts)) * 8 / (n * BH),
            "batched_scan": batched,
            **({"budget_sweep": sweep} if sweep else {}),
            **({"chan4_comparators": comparators} if comparators else {}),
            **({"klt_step": klt_step} if klt_step else {})}


class _RowsStore:
    """All layers' stores as one row set (layer-major rows), for one scan launch over every layer."""

    def __init__(self, stores):
        self.BH = sum(st.BH for st in stores)
        self.n = stores[0].n
        self.sub = stores[0].sub
        self.planes_k = torch.cat([st.planes_k for st in stores])
        self.planes32 = self.planes_k.view(torch.int32)
        self.scales_k = torch.cat([st.scales_k for st in stores])


def batched_scan_figure(a, bp, layers, n, BH, G, peaks):
    """The scan of every layer's rows in ONE launch (layer-major rows; the queries of the synthetic
    layers are independent): the kernel's throughput with enough rows to fill the machine, beside the
    per-layer launches of the decode step.  Mean per layer-equivalent over a graph of launches; inputs
    (the index of all layers, hundreds of MB) are larger than L2."""
    rs = _RowsStore([lay.store for lay in layers])
    q = torch.cat([lay.q for lay in layers])
    plan = bp.make_plan(torch.cat([lay.g for lay in layers]), a.budget)
    byts = bp.bytes_planes(plan["t"], n)
    out = torch.empty(rs.BH, G, n, device=q.device)
    reps = max(2, a.steps // 2)
    for _ in range(3):
        bp.PlaneStore.scan(rs, q, plan, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            bp.PlaneStore.scan(rs, q, plan, out=out)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    nl = len(layers)
    achieved = byts / (ms * 1e-3) / 1e9
    del g, out, rs
    torch.cuda.empty_cache()
    return {"layers_per_launch": nl, "rows_per_launch": BH * nl, "us_per_layer": ms * 1e3 / nl,
            "launch_ms": ms, "bytes_per_launch": byts,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"]}}


def scan_part(a, dev, bp, peaks):
    """--part scan (profiling): one HBM store over --scan-layers layers of the --scan-spec shape (rows
    layer-major, seeded lognormal-channel keys), 3 warm-up scans, then --steps timed scan launches over
    all rows.  An ncu capture of one launch (`-k regex:phase_scan -s 2 -c 1`) sees a launch over every
    layer's rows."""
    sp = HBM_SPECS[a.scan_spec]
    rows, G, n = sp["hkv"] * sp["batch"] * a.scan_layers, sp["g"], sp["n"]
    gen = torch.Generator(device=dev).manual_seed(5)
    scale = torch.randn(rows, 1, 128, generator=gen, device=dev).exp()
    K = torch.empty(rows, n, 128, dtype=torch.bfloat16, device=dev)
    for r0 in range(0, rows, 16):
        r1 = min(rows, r0 + 16)
        K[r0:r1] = (torch.randn(r1 - r0, n, 128, generator=gen, device=dev) * scale[r0:r1]).to(torch.bfloat16)
    q = (torch.randn(rows, G, 128, generator=gen, device=dev) * scale).contiguous()
    g = ((q ** 2) * scale ** 2).sum(1).contiguous()
    st = bp.PlaneStore(K)
    del K
    plan = bp.make_plan(g, a.budget)
    byts = bp.bytes_planes(plan["t"], n)
    out = torch.empty(rows, G, n, device=dev)
    for _ in range(3):
        st.scan(q, plan, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        st.scan(q, plan, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    return {"spec": a.scan_spec, "layers": a.scan_layers, "rows": rows, "launch_ms": ms,
            "us_per_layer": ms * 1e3 / a.scan_layers, "bytes_per_launch": byts,
            "achieved_gbs": byts / (ms * 1e-3) / 1e9, "frac_hbm": byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]}


def klt_figure(a, bp, off, layers, kvs, n, BH, k_tot, scores):
    """The same decode step over KLT-rotated stores (planesK, scripts/R_ruler.py:63-64, 82-84): per layer
    the query rotation + gains kernel, plan, scan + selection of the rotated queries, attention with the
    original ones; one CUDA graph per step.  Also the one-off store build (basis + fused rotate/quantise/
    pack) per layer."""
    from fathom_b200 import klt
    stores, builds = [], []
    for L, lay in enumerate(layers):
        K = kvs[L][0]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        basis = klt.klt_basis(K)
        if L == 0:
            torch.cuda.profiler.start()      # an ncu capture of the store-build kernel (first layer)
        e0.record()
        stores.append(klt.KLTPlaneStore(K, basis))
        e1.record()
        e1.synchronize()
        if L == 0:
            torch.cuda.profiler.stop()
        builds.append(e0.elapsed_time(e1))

    def step():
        for L, (lay, st) in enumerate(zip(layers, stores)):
            qr, gains = klt.klt_query(lay.q, st.basis)
            plan = bp.make_plan(gains, a.budget)
            idx = bp.scan_topk(st, qr, plan, k_tot, a.sink, a.local, scores=scores)
            off.decode_attention(lay.q, idx, kvs[L][0], kvs[L][1], n)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(a.warmup):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    bits = []
    for lay, st in zip(layers, stores):
        _, gains = klt.klt_query(lay.q, st.basis)
        bits.append(bp.bytes_planes(bp.make_plan(gains, a.budget)["t"], n) * 8 / (n * BH))
    del g, stores
    return {"method": f"planesK budget {a.budget:g}", "ms_per_step": ms, "bits_per_row": float(np.mean(bits)),
            "store_build_ms_per_layer": float(np.median(builds)),
            "extra_launches_per_layer": 1}


def chan4_host_figure(a, dev, bp, off, layers, kv, scores):
    """The reference's channel-subset comparators on the host-resident context of the headline step (its
    offload-table rows SparQ r = 16 and the 32-channel scan, paper/tables/tab_offload.tex): per layer the
    active channels (top-r of sum_g |q_g|, scripts/B_e2e_offload_v2.py:209), the zero-copy 4-bit scan of
    the host channel store (HostChan4Store), sink+local top-k, and the same row gather + attention as
    the bit-plane step.  4 distinct channel stores serve the layers round-robin (host memory); every
    layer scans with its own query."""
    from fathom_b200.synth import make_layer
    n, BH = a.ctx, a.hkv
    k_tot = a.k + a.sink + a.local
    stores = []
    for L in range(4):
        d = make_layer(BH, a.g, n, seed=11, layer=L, device=dev, kv_dtype=torch.bfloat16, with_v=False)
        stores.append(off.HostChan4Store(d["K"]))
        del d
    torch.cuda.empty_cache()
    out = []
    try:
        for name, r in (("sparq_r16", 16), ("channels_32", 32)):
            lists = []
            for lay in layers:
                m = torch.zeros(BH, 128, dtype=torch.bool, device=dev)
                m.scatter_(1, lay.q.abs().sum(1).topk(r, -1).indices, True)
                lists.append(m)

            def step():
                for L, lay in enumerate(layers):
                    act, nact = bp.channel_list(lists[L])
                    stores[L % len(stores)].scan(lay.q, act, nact, out=scores)
                    idx = bp.sink_local_topk(scores, k_tot, a.sink, a.local)
                    rows = kv[L % len(kv)]
                    off.decode_attention(lay.q, idx, rows["K"], rows["V"], n)

            for _ in range(a.warmup):
                step()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                step()
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / a.steps
            byts = bp.bytes_chan4(torch.full((BH,), r, dtype=torch.int32), n)
            out.append({"method": name, "bits_per_row": byts * 8 / (n * BH), "ms_per_step": ms,
                        "index_bytes_per_step": byts * len(layers),
                        "index_gbs": byts * len(layers) / (ms * 1e-3) / 1e9})
    finally:
        for st in stores:
            st.free()
    return out


def copy_index_figure(a, dev, off, layers, kv, scores):
    """The headline step with the reference's copy-index index path (offload.stream_planes,
    scripts/B_e2e_offload_v2.py:118-133, 182-196): per layer the planes and scales the plan reads are
    staged from host into device memory (SM-issued copies) chunk by chunk on a copy stream, and each
    chunk is scanned from device memory on a scan stream once it has landed; parts = 1 stages the whole
    layer before one scan.  Same selection (sink_local_topk), row gather and attention as the default
    zero-copy step, whose figure is the headline; the index bytes moved are the same."""
    k_tot = a.k + a.sink + a.local
    byts = float(np.sum([lay.bytes for lay in layers]))
    out = []
    for parts in (1, 4, 8):
        def step():
            for L, lay in enumerate(layers):
                rows = kv[L % len(kv)]
                off.decode_step(lay.q, lay.g, a.budget, lay.store, rows["K"], rows["V"], a.ctx, k_tot, a.sink,
                                a.local, scores=scores, stream_parts=parts)

        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / a.steps
        out.append({"parts": parts, "ms_per_step": ms, "index_bytes_per_step": byts,
                    "index_gbs_over_step": byts / (ms * 1e-3) / 1e9})
    off.release_staging(dev)
    return out


def chan4_figure(a, bp, layers, peaks, n, BH, scores):
    """The reference's comparator scans on the same keys (kernels/bitplane.py Chan4Store; its kernel table
    rows): SparQ r = 16 (top-16 of sum_g |q_g|), 32 channels, and the full 4-bit scan, each a graph of scans
    round-robin over 4 layers' stores (inputs larger than L2)."""
    stores = [bp.Chan4Store(lay.store_K) for lay in layers[:4]]
    out = []
    for name, r in (("sparq_r16", 16), ("channels_32", 32), ("full_4bit", 128)):
        lists = []
        for lay in layers[:4]:
            act = torch.zeros(BH, 128, dtype=torch.bool, device=lay.q.device)
            act.scatter_(1, lay.q.abs().sum(1).topk(r, -1).indices, True)
            lists.append(bp.channel_list(act))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for st, (al, nl) in zip(stores, lists):
                st.scan(layers[0].q, al, nl, out=scores)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (a.steps * len(stores))
        byts = float(np.mean([bp.bytes_chan4(nl, n) for _, nl in lists]))
        out.append({"method": name, "bits_per_row": byts * 8 / (n * BH), "scan_ms_per_layer": ms,
                    "achieved_gbs": byts / (ms * 1e-3) / 1e9, "frac_hbm": byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]})
        del g
    del stores
    return out


def hf_row_buffers(ctx, layers, hkv):
    """Distinct K/V row buffers the host can pin for the model figure: every layer's own when they fit
    in 45% of the available memory, else 4 shared round-robin (each layer still has its own index)."""
    avail = 0
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    per_layer = hkv * ctx * 512 + hkv * 128 * (-(-ctx // 64)) * 34      # rows + index
    return layers if avail == 0 or layers * per_layer <= 0.45 * avail else 4


def hf_figure(a, dev, ctxs=(262144, 524288)):
    """End-to-end decode through a Qwen3-8B-shaped transformers model (random bf16 weights: 36 layers,
    32 query / 8 KV heads, hidden 4096) whose attention is patched onto the offloaded path
    (fathom_b200.hf; scripts/B_e2e_offload_v2.py), batch 1, budget a.budget, k = a.k + sink + local,
    index and K/V rows in pinned mapped host memory.  The KV cache is synthetic (the reference's
    --synthetic-kv mode): seeded keys and values per layer, loaded and offloaded one layer at a time.
    Reported per context: wall ms per generated token with the model run eagerly (host-synchronised,
    as the reference's "wall"), wall ms per token in graph mode (OffloadedDecoder(graphs=True): one
    captured step replayed per token), and the device time of that step replayed back to back
    (launch-free, as the reference's profiler "GPU" column, paper/tables/tab_offload.tex)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from fathom_b200.hf import OffloadedDecoder
    from fathom_b200.synth import make_layer
    cfg = Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                      max_position_embeddings=1 << 21, tie_word_embeddings=False, attn_implementation="sdpa")
    old_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            torch.manual_seed(0)
            model = Qwen3ForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(old_dtype)
    k_tot = a.k + a.sink + a.local
    out = []
    for n in ctxs:
        dec = OffloadedDecoder(model, k=k_tot, sink=a.sink, local=a.local, budget=a.budget, index="host",
                               rows="host", max_new=a.local + 2 * (a.warmup + a.steps) + 8, graphs=True)
        try:
            t0 = time.time()
            nrows = hf_row_buffers(n, cfg.num_hidden_layers, cfg.num_key_value_heads)
            for L in range(cfg.num_hidden_layers):
                d = make_layer(cfg.num_key_value_heads, 4, n, seed=7, layer=L, device=dev, kv_dtype=torch.bfloat16,
                               with_v=L < nrows)
                dec.load_kv(L, d["K"].view(1, 8, n, 128), d["V"].view(1, 8, n, 128) if L < nrows else None,
                            offload=True, rows_of=None if L < nrows else L % nrows)
                del d
            build_s = time.time() - t0
            tok = torch.randint(0, cfg.vocab_size, (1, 1), device=dev)
            for _ in range(a.warmup):
                tok = dec.decode(tok).argmax(-1, keepdim=True)
            torch.cuda.synchronize(dev)
            walls = []
            for i in range(a.steps):
                if i == 0:
                    torch.cuda.profiler.start()   # `ncu --profile-from-start off` captures this one eager step
                t1 = time.perf_counter()
                tok = dec.decode(tok).argmax(-1, keepdim=True)
                torch.cuda.synchronize(dev)
                walls.append((time.perf_counter() - t1) * 1e3)
                if i == 0:
                    torch.cuda.profiler.stop()
            wall = float(np.median(walls))
            # graph mode: eager steps until the local window lies in the recent buffer, then one captured
            # step replayed per token (OffloadedDecoder(graphs=True)); wall per token, host-synchronised
            while dec.cache[0].nrec + 1 < a.local:
                tok = dec.decode(tok).argmax(-1, keepdim=True)
            for _ in range(a.warmup):
                tok = dec.decode(tok).argmax(-1, keepdim=True)
            torch.cuda.synchronize(dev)
            gwalls = []
            for _ in range(a.steps):
                t1 = time.perf_counter()
                tok = dec.decode(tok).argmax(-1, keepdim=True)
                torch.cuda.synchronize(dev)
                gwalls.append((time.perf_counter() - t1) * 1e3)
            graph_wall = float(np.median(gwalls))
            # device time of one step: the captured graph replayed back to back
            g = dec._graph
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            gpu_ms = e0.elapsed_time(e1) / a.steps
            graph_note = None
            out.append({"ctx": n, "wall_ms_per_token": wall, "tok_per_s": 1e3 / wall,
                        "graph_wall_ms_per_token": graph_wall, "tok_per_s_graph": 1e3 / graph_wall,
                        "gpu_ms_per_token": gpu_ms, "tok_per_s_gpu": (1e3 / gpu_ms) if gpu_ms else None,
                        "offload_build_s": build_s, "row_buffers": nrows,
                        **({"note": graph_note} if graph_note else {})})
        finally:
            dec.free()
            dec.unpatch()
            torch.cuda.empty_cache()
    del model
    torch.cuda.empty_cache()
    return {"model": "Qwen3-8B shape, random bf16 weights", "batch": 1, "budget": a.budget, "k": k_tot,
            "index": "host", "rows": "host", "kv": "synthetic (seeded per layer)", "per_ctx": out}


# ------------------------------------------------------------------ multi-GPU figures (N > 1)
def free_host_layers(layers, kv):
    """Releases the pinned host memory of a rank's index layers and K/V row buffers."""
    seen = set()
    for lay in layers:
        if id(lay.store) not in seen:
            seen.add(id(lay.store))
            lay.store.free()
    for rows in kv:
        for buf in rows["bufs"]:
            buf.free()
    layers.clear()
    kv.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def sharded_parity(a, layers, scores, rank, world, bp):
    """Bit-exactness of the NCCL merge on this run's own data: layer 0's context-sharded selection (local
    top-k per rank, all-gather, merge) against one selection over the whole context, whose scores are
    the ranks' chunks all-gathered (per-token scores do not depend on the chunking: chunks are
    64-token aligned).  True on every rank, or False."""
    from fathom_b200 import shard
    lay = layers[0]
    n_total = a.ctx * world
    lo, hi = rank * a.ctx, (rank + 1) * a.ctx
    plan = bp.make_plan(lay.g, a.budget)
    mlo, mhi = shard.local_window(lo, hi, n_total, a.sink, a.local)
    idx_l, vals_l, _ = bp.scan_select(lay.store, lay.q, plan, a.k, mask_lo=mlo, mask_hi=mhi, index_offset=lo,
                                      scores=scores, with_scores=True)
    top = shard.merge_shards(idx_l, vals_l, a.k)
    ok = shard.merged_equals_single(scores, top, n_total, a.k, a.sink, a.local)
    t = torch.tensor([1 if ok else 0], device=scores.device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
    return {"merged_indices_equal": bool(t.item()), "layer": 0, "rows": int(top.shape[0] * top.shape[1]),
            "ctx_total": n_total, "k": a.k,
            "check": "merged top-k of the ranks' local selections (NCCL all-gather + merge) equals one selection "
                     "over all ranks' all-gathered score chunks, order included"}


def timed_sharded_steps(b, layers, kv, scores, rank, world, dev):
    """Warm-up and timed context-sharded decode steps; ms per step, max over ranks."""
    from fathom_b200 import shard
    outs = [None] * len(layers)
    for _ in range(b.warmup):
        shard.sharded_decode_step(b, layers, kv, scores, outs, rank, world)
    torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(b.steps):
        shard.sharded_decode_step(b, layers, kv, scores, outs, rank, world)
    e1.record()
    torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / b.steps], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


CONFIG4_CTX = 4194304


def config4_figure(a, kv_arg, dev, bp, off, rank, world):
    """Config 4 as stated: one sequence of 4,194,304 tokens split into contiguous chunks over the ranks
    (strong scaling), index and K/V rows host-resident, each rank scanning its chunk through its own
    host link, local top-k, NCCL all-gather + merge, partial attention + combine."""
    import copy
    b = copy.copy(a)
    b.ctx = CONFIG4_CTX // world
    b.kv_buffers = kv_arg
    t0 = time.time()
    layers, kv = build_host_layers(b, dev, rank, world, bp, off)
    build_s = time.time() - t0
    scores = torch.empty(b.hkv, b.g, b.ctx, device=dev)
    try:
        ms = timed_sharded_steps(b, layers, kv, scores, rank, world, dev)
        parity = sharded_parity(b, layers, scores, rank, world, bp)
    finally:
        free_host_layers(layers, kv)
    rows = CONFIG4_CTX * b.hkv * b.layers
    return {"workload": "config4: one sequence of 4,194,304 tokens, contiguous chunks per GPU (strong scaling), "
                        "host-resident index + K/V rows, NCCL merge", "scaling": "strong",
            "ctx_total": CONFIG4_CTX, "ctx_per_gpu": b.ctx, "value": rows / (ms * 1e-3), "unit": "key-rows/s",
            "ms_per_step": ms, "index_buffers": b.index_buffers, "kv_row_buffers": b.kv_buffers,
            "build_s": build_s, "merged_indices_equal": parity["merged_indices_equal"]}


def config3_replicas(a, dev, bp, off, peaks, rank, world):
    """Config 3 on N GPUs: the 8 independent sequences split 8/N per GPU (replicas, no collective in the
    step); the aggregate is all sequences' key rows over the slowest rank's step."""
    fig = hbm_figure(a, dev, bp, off, peaks, "config3", batch=HBM_SPECS["config3"]["batch"] // world, seed=3 + 17 * rank)
    t = torch.tensor([fig["ms_per_step"], fig["scan_ms_per_layer"]], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, scan_ms = t.tolist()
    sp = HBM_SPECS["config3"]
    rows = sp["n"] * sp["hkv"] * sp["batch"] * sp["layers"]
    return {"workload": sp["workload"] + f"; {sp['batch'] // world} sequence(s) per GPU", "scaling": "replicas",
            "value": rows / (ms * 1e-3), "unit": "key-rows/s", "ms_per_step": ms, "scan_ms_per_layer": scan_ms,
            "sequences_per_gpu": sp["batch"] // world}


# ------------------------------------------------------------------ main
def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    from fathom_b200 import bitplane as bp
    from fathom_b200 import offload as off
    from fathom_b200 import _lib
    _lib.lib()
    peaks, peaks_kind = measured_peaks()
    if a.part == "hbm":
        if rank == 0:
            print(json.dumps({"hbm_resident": hbm_figure(a, dev, bp, off, peaks)}), flush=True)
        return
    if a.part == "config3":
        if rank == 0:
            print(json.dumps({"batched_hbm": hbm_figure(a, dev, bp, off, peaks, "config3")}), flush=True)
        return
    if a.part == "scan":
        if rank == 0:
            print(json.dumps({"scan": scan_part(a, dev, bp, peaks)}), flush=True)
        return
    if a.part == "hf":
        if rank == 0:
            ctxs = tuple(int(x) for x in a.hf_ctx.split(",")) if a.hf_ctx else (262144, 524288, 1048576)
            print(json.dumps({"hf_decode": hf_figure(a, dev, ctxs)}), flush=True)
        return

    link, link_ranks = probe_gbs(LinkProbe(dev), world)
    sm_read, sm_read_ranks = probe_gbs(SMReadProbe(dev, off), world)
    log(f"[rank {rank}] SM reads of mapped host memory {sm_read:.1f} GB/s (all ranks at once; per rank {sm_read_ranks})")
    log(f"[rank {rank}] host link H2D {link:.1f} GB/s (all ranks at once; per rank {link_ranks})")
    t0 = time.time()
    kv_arg = a.kv_buffers                       # build_host_layers lowers a.kv_buffers to what host memory holds
    layers, kv = build_host_layers(a, dev, rank, world, bp, off)
    log(f"[rank {rank}] built {a.layers} host layers in {time.time() - t0:.1f} s")
    scores = torch.empty(a.hkv, a.g, a.ctx, device=dev)
    outs = [None] * a.layers

    if world > 1:
        from fathom_b200 import shard
        step_fn = lambda q_in=None, g_in=None, ev=None: shard.sharded_decode_step(
            a, layers, kv, scores, outs, rank, world, q_in=q_in, g_in=g_in, scan_events=ev)
    else:
        step_fn = lambda q_in=None, g_in=None, ev=None: decode_step_1gpu(
            a, layers, kv, bp, off, scores, outs, q_in=q_in, g_in=g_in, scan_events=ev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(a.warmup):
        step_fn()
    barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    ev = []
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()        # `ncu --profile-from-start off` captures the timed steps only
    e0.record()
    for _ in range(a.steps):
        step_fn(ev=ev)
    e1.record()
    barrier()
    torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1) / a.steps

    # e2e through the public API with host buffers: H2D of the step's q/g, D2H of the outputs
    q_host = torch.stack([l.q for l in layers]).cpu().pin_memory()
    g_host = torch.stack([l.g for l in layers]).cpu().pin_memory()
    out_host = torch.empty(a.layers, a.hkv, a.g, 128, pin_memory=True)
    q_dev = torch.empty_like(q_host, device=dev)
    g_dev = torch.empty_like(g_host, device=dev)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(a.steps):
        q_dev.copy_(q_host, non_blocking=True)
        g_dev.copy_(g_host, non_blocking=True)
        step_fn(q_in=q_dev, g_in=g_dev)
        out_host.copy_(torch.stack(outs), non_blocking=True)
    f1.record()
    barrier()
    clk = clocks.stop()
    e2e_ms = f0.elapsed_time(f1) / a.steps

    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    rows_step = a.ctx * world * a.hkv * a.layers
    durs = [x.elapsed_time(y) for x, y, _ in ev]
    byts = [b for _, _, b in ev]
    scan_ms = float(np.mean(durs))
    achieved = float(np.mean(byts)) / (scan_ms * 1e-3) / 1e9
    per_rank_achieved = [achieved]
    if world > 1:          # every rank's scan ran at the same time: the aggregate is the sum
        per_rank_achieved = shard.all_gather(torch.tensor([achieved], device=dev, dtype=torch.float64)).flatten().tolist()
        achieved = float(sum(per_rank_achieved))
    bits_row = float(np.mean(byts)) * 8 / (a.ctx * a.hkv)
    # plan, scan, group-key selection, dedupe, gather, attend; sharded: + merge, combine
    launches_per_layer = 6 if world == 1 else 8
    line = {"metric": METRIC, "value": rows_step / (ms * 1e-3), "unit": "key-rows/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "decode_step_us": ms * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded lognormal-channel keys/values/queries)", "config": config_dict(a, world),
            "bits_per_row": bits_row,
            "roofline": {"bound": "host_link", "achieved": achieved, "peak": link, "unit": "GB/s",
                         "frac": achieved / link, "traffic": float(np.mean(byts)) * TRAFFIC_RATIO_HOST,
                         "traffic_source": "ncu pcie__read_bytes.sum per launch, T=262144 capture scaled by units",
                         "bytes_per_launch": float(np.mean(byts)),
                         "kernel": "scan (zero-copy reads of the host index)",
                         "peak_source": "pinned H2D cudaMemcpy of 1 GiB measured in this run" + (
                             "" if world == 1 else ", on every rank at once (barrier-synchronised rounds): all "
                                                   "ranks' bytes over the slowest rank's time; achieved is the sum "
                                                   "of the ranks' concurrent scan rates"),
                         "sm_read_gbs": sm_read, "frac_of_sm_read": achieved / sm_read,
                         "sm_read_source": "element-wise kernel reading 1 GiB of mapped host memory, this run "
                                           "(the ceiling of GPU-issued zero-copy reads; the DMA copy above is higher)"
                                           + ("" if world == 1 else ", on every rank at once"),
                         **({} if world == 1 else {"per_rank_achieved": per_rank_achieved,
                                                   "per_rank_link_gbs": link_ranks,
                                                   "per_rank_sm_read_gbs": sm_read_ranks})},
            "scan_ms_per_layer": scan_ms,
            "e2e": {"value": rows_step / (e2e_ms * 1e-3), "unit": "key-rows/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": q_host.numel() * 4 + g_host.numel() * 4,
                    "d2h_bytes_per_step": out_host.numel() * 4},
            "gpu_launches": launches_per_layer * a.layers * a.steps,
            "clocks": clk, "peaks_source": peaks_kind}
    if world > 1:
        # every rank takes part in each of these (collectives inside); rank 0 reports them
        line["parity"] = sharded_parity(a, layers, scores, rank, world, bp)
        free_host_layers(layers, kv)
        if a.part == "all":
            line["config4"] = config4_figure(a, kv_arg, dev, bp, off, rank, world)
            line["config3_replicas"] = config3_replicas(a, dev, bp, off, peaks, rank, world)
    if rank == 0 and world == 1 and not a.no_hbm and a.part == "all":
        try:
            line["copy_index_host"] = copy_index_figure(a, dev, off, layers, kv, scores)
        except Exception as exc:                          # the headline line stands without this figure
            line["copy_index_host"] = {"error": f"{type(exc).__name__}: {str(exc)[:200]}"}
        try:
            line["chan4_host"] = chan4_host_figure(a, dev, bp, off, layers, kv, scores)
        except Exception as exc:                          # the headline line stands without this figure
            line["chan4_host"] = {"error": f"{type(exc).__name__}: {str(exc)[:200]}"}
        del layers, kv
        torch.cuda.empty_cache()
        line["hbm_resident"] = hbm_figure(a, dev, bp, off, peaks)
        line["batched_hbm"] = hbm_figure(a, dev, bp, off, peaks, "config3")
    if rank == 0 and world == 1 and not a.no_hf and a.part == "all":
        try:
            line["hf_decode"] = hf_figure(a, dev, ctxs=(262144, 1048576))
        except Exception as exc:                          # the headline line stands without this figure
            line["hf_decode"] = {"error": f"{type(exc).__name__}: {str(exc)[:200]}"}
    if rank == 0 and world == 1 and not a.no_cpu and a.part == "all":
        t, r = cpu_sample(a, a.cpu_heads)
        line["cpu_baseline"] = {"value": r / t, "unit": "key-rows/s", "cores": os.cpu_count(), "kind": "port",
                                "cpu_model": cpu_model(),
                                "sample": f"{a.cpu_heads} KV heads x {a.ctx} tokens of one layer: plan+scan+"
                                          f"sink_local_topk+attention, numpy oracle restatement with the scan on a "
                                          f"{os.cpu_count()}-thread pool ({t:.1f} s)"}
    if rank == 0:
        # bounded device waits that gave up during the run (NaN-scored tiles); 0 in a valid run
        import ctypes
        from fathom_b200 import _lib
        count = ctypes.c_ulonglong(0)
        _lib.check(_lib.lib().fathom_wait_timeouts(ctypes.byref(count), 0), "wait_timeouts")
        line["wait_timeouts"] = int(count.value)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
