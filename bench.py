"""Benchmark of the routed-MoE expert-offload hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload decode|fetch|prefill|ep|ep-rank|layer] [--impl ours|reference]

Workloads:

* ``decode`` (default) -- configs[2]: 40-layer Drama-3-shaped MoE decode,
  batch 1, random init (hidden 2048, 256 experts, top-8, FP8 experts + 6.9 GiB
  of bf16 dense weights read per token), experts offloaded to pinned host
  memory with an 8 GiB device cache (68 slots per layer), routing from the
  seeded Zipf(1.1) trace.  One step = one token through all 40 layers, replayed
  from a CUDA graph.  Metric: decode tok/s; the fetch kernel's host-link GB/s
  against the measured pinned copy-engine peak is reported beside it.
* ``fetch`` -- configs[1]: the expert-fetch microbenchmark (40 x 256 experts
  pinned, 2048 slots in total, graph-captured allocator + fetch per layer).
* ``prefill`` -- configs[3]: a 2048-token chunk through 40 offloaded layers
  (union gather + token-permuted FP8 grouped GEMM).
* ``ep`` -- configs[4]: resident expert-parallel decode, batch 64, 256 experts
  sharded over N GPUs, NCCL all-to-all dispatch/combine.
* ``layer`` -- configs[0]: one MoE layer over 16 tokens with 256 resident
  experts, the CPU restatement timed beside it.
* ``ep-rank`` -- configs[4], one rank: the expert call of an N-GPU
  expert-parallel step (``--ep-ranks N``: 256/N local experts, the rank's
  received rows) on one GPU, through the folded NVLink call on a local
  stand-in of the link; the per-rank roofline at every N without N GPUs.

Inputs are far larger than L2 (30 GiB host store, 6.9 GiB dense weights, 8 GiB
cache).  Multi-GPU runs are replicas (each rank its own store, cache and host
link; "scaling": "weak"), timed on the device, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

EXPERT_BYTES = 3_146_496
METRIC_DECODE = "decode tok/s (40L, bs1, offloaded) + expert-fetch GB/s vs host-link peak"
METRIC_FETCH = "expert-fetch GB/s (40L x 256 experts pinned, 2048-slot cache, Zipf(1.1), graph)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "fetch", "ep", "ep-rank", "prefill", "layer"),
                    default="decode")
    ap.add_argument("--ep-ranks", type=int, default=8,
                    help="ep-rank workload: the N whose per-rank expert call is emulated")
    ap.add_argument("--prefill-tokens", type=int, default=2048)
    ap.add_argument("--no-prefetch", action="store_true",
                    help="prefill: gather each layer's union after its router (no gather of the "
                         "next layer during this layer's GEMM)")
    ap.add_argument("--global-batch", type=int, default=64, help="ep workload: decode streams")
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--slots", type=int, default=2048, help="fetch workload: slots over all layers")
    ap.add_argument("--cache-gib", type=float, default=8.0, help="decode workload device cache")
    ap.add_argument("--policy", choices=("lru", "lfu"), default="lru")
    ap.add_argument("--no-overlap", action="store_true",
                    help="decode: separate fetch and gate/up launches")
    ap.add_argument("--one-host-copy", action="store_true",
                    help="decode: one copy of the host store for all local ranks instead of "
                         "one per NUMA node of their GPUs")
    ap.add_argument("--l2-warm-mib", type=float, default=85.0,
                    help="decode: MiB of the next layer's first dense weight hinted into L2 "
                         "during each layer's fetch (85 = all of it; 0 = off)")
    ap.add_argument("--no-l2-warm-gate", action="store_true",
                    help="decode: do not hint the next layer's router gate weight into L2")
    ap.add_argument("--fetch-ctas", type=int, default=0)
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    ap.add_argument("--cpu-layers", type=int, default=8,
                    help="decode CPU legs: layers per sampled token (time scaled to --layers)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=0,
                    help="decode: end-to-end steps (0 = --steps, the timed window)")
    ap.add_argument("--cache-warm-steps", type=int, default=512,
                    help="decode: graph replays that bring the caches to steady state "
                         "before --warmup")
    ap.add_argument("--ep-exchange", choices=("p2p", "nccl"), default="p2p",
                    help="ep workload: NVLink peer stores or NCCL all-to-all")
    ap.add_argument("--no-ep", action="store_true",
                    help="decode: skip the resident expert-parallel sub-record")
    return ap.parse_args()


def init_dist(args):
    from drama3_offloading_b200.benchutil import dist_env
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    return rank, world, local


def local_group(world):
    """Process group of this machine's ranks (single-node runs: all ranks)."""
    if world <= 1:
        return None
    import torch.distributed as dist
    return dist.group.WORLD


# ---------------------------------------------------------------- CPU legs (oracle)

class CpuDecodeSample:
    """``layers`` CPU layers of the decode stack: torch bf16 dense GEMVs, the
    oracle router, the oracle LRU allocator, a memcpy of each missed expert
    into a host-side cache, and the oracle's dequantise-then-matmul experts
    (the reference's torch CPU MoE path).  A bounded sample of the 40 layers."""

    def __init__(self, layers, trace, capacity, hidden=2048, inter=512, experts=256, R=None,
                 seed=0):
        import oracle
        from drama3_offloading_b200 import synth
        self.o = oracle
        torch.set_num_threads(os.cpu_count() or 1)
        self.threads = torch.get_num_threads()
        gen = "cuda" if torch.cuda.is_available() else "cpu"
        g = torch.Generator().manual_seed(seed + 7)
        self.L, self.k, self.trace = layers, trace.shape[2], trace
        from drama3_offloading_b200 import decode as dec
        if R is None:  # the GPU stack's dense stand-in rows (6.9 GiB with the shared experts)
            R = dec.dense_stand_in_rows(40, hidden, inter, dec.DENSE_GIB)
        # the full-attention layers' 2048-token KV context, as on the GPU
        self.kv = {l: ((torch.randn(dec.KV_HEADS, dec.KV_CONTEXT, dec.HEAD_DIM, generator=g)
                        * 0.5).to(torch.bfloat16),
                       torch.randn(dec.KV_HEADS, dec.KV_CONTEXT, dec.HEAD_DIM, generator=g)
                       .to(torch.bfloat16))
                   for l in dec.full_attention_layers(layers)}
        self.head_dim = dec.HEAD_DIM
        self.ex = [synth.make_experts(experts, hidden, inter, seed=seed + l, device=gen,
                                      chunk=32).to("cpu") for l in range(layers)]
        self.up = [(torch.randn(R, hidden, generator=g) * hidden ** -0.5).to(torch.bfloat16)
                   for _ in range(layers)]
        self.down = [(torch.randn(hidden, R, generator=g) * (R ** -0.5 * 0.5)).to(torch.bfloat16)
                     for _ in range(layers)]
        self.gate = [(torch.randn(experts, hidden, generator=g) * 0.02).to(torch.bfloat16)
                     for _ in range(layers)]
        self.shared = [((torch.randn(2 * inter, hidden, generator=g) * 0.02).to(torch.bfloat16),
                        (torch.randn(hidden, inter, generator=g) * 0.02).to(torch.bfloat16),
                        (torch.randn(hidden, generator=g) * 0.02).to(torch.bfloat16))
                       for _ in range(layers)]
        self.tabs = [oracle.init_tables(experts, capacity) for _ in range(layers)]
        self.c13 = [torch.zeros((capacity, 2 * inter, hidden), dtype=torch.float8_e4m3fn)
                    for _ in range(layers)]
        self.c2 = [torch.zeros((capacity, hidden, inter), dtype=torch.float8_e4m3fn)
                   for _ in range(layers)]
        self.s13 = [torch.ones(capacity, 2 * inter // 128, hidden // 128) for _ in range(layers)]
        self.s2 = [torch.ones(capacity, hidden // 128, inter // 128) for _ in range(layers)]
        self.h = torch.randn(1, hidden, generator=g).to(torch.bfloat16)
        self.pos = 0

    def token(self) -> float:
        o = self.o
        t0 = time.perf_counter()
        row = self.trace[self.pos % self.trace.shape[0]]
        for l in range(self.L):
            h = self.h
            h = h + torch.nn.functional.silu(h @ self.up[l].t()) @ self.down[l].t()
            if l in self.kv:
                kc, vc = self.kv[l]
                q = h.view(kc.shape[0], -1, self.head_dim)
                pr = torch.softmax(torch.bmm(q, kc.transpose(1, 2)).float()
                                   * self.head_dim ** -0.5, dim=-1).to(torch.bfloat16)
                h = h + 0.25 * torch.bmm(pr, vc).view(1, -1)
            _, w, _, _ = o.router_topk(h, self.gate[l], self.k)
            ys = o.shared_expert_forward(h, *self.shared[l])
            slots, fs, fe, n = o.resolve(self.tabs[l], row[l])
            ex = self.ex[l]
            for j in range(n):
                s, e = int(fs[j]), int(fe[j])
                self.c13[l][s].copy_(ex.w13_weight[e])
                self.c2[l][s].copy_(ex.w2_weight[e])
                self.s13[l][s].copy_(ex.w13_scale_inv[e])
                self.s2[l][s].copy_(ex.w2_scale_inv[e])
            y = o.moe_forward(h, torch.from_numpy(slots.astype(np.int64)).reshape(1, -1), w,
                              self.c13[l], self.s13[l], self.c2[l], self.s2[l])
            y = h.float() + y + ys
            y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)
            self.h = y.to(torch.bfloat16)
        self.pos += 1
        return time.perf_counter() - t0


def cpu_decode_baseline(trace, capacity, layers_total, sample_layers, sample_s) -> dict:
    cpu = CpuDecodeSample(sample_layers, trace, capacity)
    cpu.token()  # warm
    t0 = time.perf_counter()
    times = []
    while time.perf_counter() - t0 < sample_s or not times:
        times.append(cpu.token())
    per_layer = float(np.mean(times)) / sample_layers
    return {"value": 1.0 / (per_layer * layers_total), "unit": "tok/s", "cores": cpu.threads,
            "kind": "port",
            "sample": f"{len(times)} tokens x {sample_layers} of {layers_total} layers (per-token "
                      f"time scaled by {layers_total}/{sample_layers}); torch bf16 dense GEMVs + "
                      f"oracle router/LRU + expert memcpy + dequantised fp32 expert matmuls + "
                      f"shared expert + KV-context attention on the full-attention layers"}


def cpu_fetch_baseline(trace, capacity, sample_s) -> dict:
    """The oracle allocator + a memcpy of every missed expert (host store ->
    host cache), one thread, over a bounded prefix of the trace."""
    import oracle
    layers = trace.shape[1]
    store = np.random.default_rng(0).integers(0, 255, size=(16, EXPERT_BYTES), dtype=np.uint8)
    cache = np.zeros((capacity, EXPERT_BYTES), dtype=np.uint8)
    tabs = [oracle.init_tables(256, capacity) for _ in range(layers)]
    t0 = time.perf_counter()
    steps = misses = 0
    while time.perf_counter() - t0 < sample_s and steps < trace.shape[0]:
        for l in range(layers):
            _, fs, fe, n = oracle.resolve(tabs[l], trace[steps, l])
            for j in range(n):
                cache[fs[j]] = store[int(fe[j]) % 16]
            misses += n
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": misses * EXPERT_BYTES / dt / 1e9, "unit": "GB/s", "cores": 1,
            "kind": "port",
            "sample": f"first {steps} steps x {layers} layers of the Zipf trace: LRU oracle + memcpy "
                      f"of each missed 3,146,496-B expert (host->host)"}


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------- decode

def decode_config(args, capacity: int | None = None) -> dict:
    """The decode workload's ``config`` (the same dict for both arms)."""
    from drama3_offloading_b200 import decode as dec
    cap = capacity or max(1, int(args.cache_gib * (1 << 30)) // (args.layers * EXPERT_BYTES))
    dense = dec.dense_bytes_per_token(args.layers)
    return {"workload": "decode-40L-bs1-offloaded", "layers": args.layers, "hidden": 2048,
            "experts": 256, "topk": 8, "shared_expert": True, "cache_gib": args.cache_gib,
            "slots_per_layer": cap, "policy": args.policy, "fetch_overlap": not args.no_overlap,
            "kv_context": dec.KV_CONTEXT, "l2_warm_mib": args.l2_warm_mib,
            "l2_warm_gate": not args.no_l2_warm_gate,
            "kv_mib_per_token": len(dec.full_attention_layers(args.layers)) * 2 *
            dec.KV_CONTEXT * dec.KV_HEADS * dec.HEAD_DIM * 2 / 2**20,
            "dense_gib_per_token": dense / 2**30,
            "cache_warm_steps": args.cache_warm_steps,
            "l2": "inputs > L2 (30 GiB host store, 6.9 GiB dense, 8 GiB cache)",
            "parallelism": f"replicas{args.gpus}"}


# PCIe read bytes per missed expert of the overlapped fetch launch
# (fetch_gemv13_kernel), from one ncu capture of the 4-layer decode case:
# pcie__read_bytes.sum of the 16 captured launches (120,489,472 B) / the 35
# experts they fetched (profiles/fetch_gemv13_kernel_traffic_decode4L.md):
# 1.094 x the 3,146,496 algorithmic bytes (the 12-byte completion header of
# every 128-byte read request counts as read traffic).
FETCH_PCIE_BYTES_PER_EXPERT = 3_442_556


def run_decode(args, rank, world, local):
    """configs[2].  After capture the caches are warmed to steady state by
    ``--cache-warm-steps`` graph replays plus the ``--warmup`` ones; the
    state at the start of the timed window is then snapshotted, so the end-to-
    end run and the fetch-kernel timing replay exactly the same window of
    tokens from exactly the same cache state as the device-timed ``value``."""
    from drama3_offloading_b200 import benchutil
    from drama3_offloading_b200.decode import DecodeStack

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak = benchutil.host_link_peak_gbs(device=dev)
    # one shared host store per machine; each replica walks the trace from
    # its own offset (independent token streams)
    stack = DecodeStack(layers=args.layers, cache_gib=args.cache_gib, device=dev,
                        policy=args.policy, group=local_group(world), local_rank=local,
                        trace_offset=512 * rank, overlap=not args.no_overlap,
                        host_per_node=not args.one_host_copy, l2_warm_mib=args.l2_warm_mib,
                        l2_warm_gate=not args.no_l2_warm_gate)
    from drama3_offloading_b200 import devcache
    devcache.FETCH_CTAS = args.fetch_ctas
    if args.fetch_ctas > 0:
        devcache.OVERLAP_FETCH_CTAS = args.fetch_ctas
    g = stack.capture()
    for _ in range(args.cache_warm_steps + args.warmup):
        g.replay()
    window = stack.snapshot()
    c0 = stack.store.counters()
    benchutil.barrier(world, dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    ms = a.elapsed_time(b)
    c1 = stack.store.counters()
    misses = (c1["misses"] - c0["misses"]) / args.steps
    hits = (c1["hits"] - c0["hits"]) / args.steps
    ms_max = benchutil.max_over_ranks(ms, world, dev)
    value = world * args.steps / (ms_max * 1e-3)

    # end to end through the public API, the same window from the same state:
    # per token the input hidden state comes from pinned host memory and the
    # output goes back to it before the next token starts
    e2e_steps = args.e2e_steps or args.steps
    stack.restore(window)
    h_in = window["h"].cpu().pin_memory()
    h_out = torch.empty(1, stack.H, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        stack.h.copy_(h_in, non_blocking=True)
        g.replay()
        h_out.copy_(stack.h, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        h_in.copy_(h_out)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = benchutil.max_over_ranks(e0.elapsed_time(e1), world, dev)
    e2e = world * e2e_steps / (e2e_ms * 1e-3)

    # the fetch launch's bandwidth over the same window again: eager steps
    # with CUDA events around every layer's fetch launch
    stack.restore(window)
    ft = stack.sample_fetch_timing(args.steps)
    fetch_gbs = ft["bytes"] / (ft["ms"] * 1e-3) / 1e9 if ft["ms"] > 0 else 0.0
    hs = stack.store.host
    host_store = {"copies": hs.copies, "gpu_nodes": [hs.rank_nodes[r] for r in sorted(hs.rank_nodes)],
                  "node": hs.node, "bound": bool(hs.bound)}
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([fetch_gbs, float(bool(hs.bound))], dtype=torch.float64, device=dev)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        host_store["fetch_gbs_per_rank"] = [round(float(x[0]), 2) for x in out]
        host_store["bound_per_rank"] = [bool(x[1]) for x in out]
    hbm = measured_peaks()
    roof_ms = stack.roofline_ms(hits, misses, hbm["hbm_gbs"], peak["gbs"])
    return {"value": value, "ms": ms_max, "e2e": e2e, "e2e_steps": e2e_steps,
            "clk": clk.summary(), "peak": peak,
            "hits": hits, "misses": misses, "fetch_gbs": fetch_gbs, "fetch_sample": ft,
            "roof_ms": roof_ms, "hbm": hbm, "capacity": stack.capacity,
            "launches": stack.launches_per_step() * args.steps, "trace": stack.trace_dev.cpu().numpy(),
            "dense_bytes": stack.dense_bytes, "host_store": host_store}


# ---------------------------------------------------------------- fetch

def run_fetch(args, rank, world, local):
    from drama3_offloading_b200 import benchutil, devcache
    from drama3_offloading_b200.stack import OffloadedExperts
    from drama3_offloading_b200.trace import zipf_trace

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    capacity = max(1, args.slots // args.layers)
    steps_total = 4096
    trace = zipf_trace(steps=steps_total, layers=args.layers)
    peak = benchutil.host_link_peak_gbs(device=dev)
    store = OffloadedExperts(layers=args.layers, capacity=capacity, device=dev,
                             policy=args.policy, fill="random", group=local_group(world),
                             local_rank=local)
    devcache.FETCH_CTAS = args.fetch_ctas
    trace_dev = torch.from_numpy(trace.astype(np.int32)).to(dev)
    step_idx = torch.zeros(1, dtype=torch.int64, device=dev)

    def one_step():
        cur = trace_dev.index_select(0, step_idx)[0]
        step_idx.add_(1).remainder_(steps_total)
        for l, ex in enumerate(store.layers):
            devcache.dev_resolve_and_fetch(ex, cur[l])

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        one_step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        one_step()
    store.reset_caches()
    step_idx.zero_()
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    c0 = store.counters()
    benchutil.barrier(world, dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    ms = a.elapsed_time(b)
    c1 = store.counters()
    misses = c1["misses"] - c0["misses"]
    hits = c1["hits"] - c0["hits"]
    fetched = c1["bytes_fetched"] - c0["bytes_fetched"]
    ms_max = benchutil.max_over_ranks(ms, world, dev)
    total_bytes = benchutil.sum_over_ranks(fetched, world, dev)
    return {"value": total_bytes / (ms_max * 1e-3) / 1e9, "ms": ms_max,
            "gbs_rank": fetched / (ms * 1e-3) / 1e9, "peak": peak, "clk": clk.summary(),
            "hit_rate": hits / max(1, hits + misses), "misses_per_step": misses / args.steps,
            "capacity": capacity, "trace": trace, "launches": args.steps * args.layers * 2}


# ---------------------------------------------------------------- prefill

def run_prefill(args, rank, world, local):
    """Prefill gather: a 2048-token bf16 chunk through 40 offloaded layers; per
    layer the router runs, the union of routed experts (top-8 per token under a
    Zipf(1.1) prior) is gathered -- cached ones borrowed read-only from the
    decode cache, the rest fetched from pinned host -- and the token-permuted
    FP8 grouped GEMM runs on the compact set.  One chunk per step, graph-
    captured; caches warmed by 64 decode steps of the Zipf trace first."""
    from drama3_offloading_b200 import benchutil, devcache, moe, offload
    from drama3_offloading_b200.stack import OffloadedExperts
    from drama3_offloading_b200.trace import zipf_trace

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T = args.prefill_tokens
    peak = benchutil.host_link_peak_gbs(device=dev)
    cap = max(1, int(args.cache_gib * (1 << 30)) // (args.layers * EXPERT_BYTES))
    store = OffloadedExperts(layers=args.layers, capacity=cap, device=dev, policy=args.policy,
                             group=local_group(world), local_rank=local)
    dec = torch.from_numpy(zipf_trace(steps=64, layers=args.layers).astype(np.int32)).to(dev)
    for s in range(64):
        for l, ex in enumerate(store.layers):
            devcache.dev_resolve_and_fetch(ex, dec[s, l])
    pre = zipf_trace(steps=T, layers=args.layers, seed=1 + rank)       # [T, L, 8]
    ids = torch.from_numpy(np.ascontiguousarray(pre.transpose(1, 0, 2)).astype(np.int32)).to(dev)
    g = torch.Generator(device=dev).manual_seed(3)
    gate = [(torch.randn(256, 2048, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            for _ in range(args.layers)]
    h0 = torch.randn(T, 2048, generator=g, device=dev).to(torch.bfloat16)
    h = h0.clone()
    wts = torch.empty(T, 8, dtype=torch.float32, device=dev)
    rids = torch.empty(T, 8, dtype=torch.int32, device=dev)

    pf = None if args.no_prefetch else offload.ChunkPrefetch(store.layers, dev)

    def step(events=None):
        h.copy_(h0)
        for l, ex in enumerate(store.layers):
            moe.router_topk(h, gate[l], 8, out_ids=rids, out_w=wts)
            if events is not None:
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
            y = (offload.offloaded_forward(ex, h, ids[l], wts) if pf is None
                 else pf.forward(l, h, ids[l], wts))
            if events is not None:
                e1.record()
                events.append((e0, e1))
            h.add_(y)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step()
    for _ in range(args.warmup):
        gr.replay()
    torch.cuda.synchronize(dev)
    c0 = [offload.gather_counters(ex) for ex in store.layers]
    benchutil.barrier(world, dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            gr.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    ms = benchutil.max_over_ranks(a.elapsed_time(b), world, dev)
    c1 = [offload.gather_counters(ex) for ex in store.layers]
    fetched = sum(x["gather_misses"] - y["gather_misses"] for x, y in zip(c1, c0)) / args.steps
    borrowed = sum(x["gather_hits"] - y["gather_hits"] for x, y in zip(c1, c0)) / args.steps
    fetch_gbs = fetched * EXPERT_BYTES / (ms / args.steps * 1e-3) / 1e9
    evs = []
    step(evs)
    torch.cuda.synchronize(dev)
    layer_ms = sum(x.elapsed_time(y) for x, y in evs)
    flops = T * 8 * 6_291_456 * args.layers
    return {
        "metric": "prefill tok/s (2048-token chunk, 40L, offloaded, union gather + FP8 grouped GEMM)",
        "value": world * T * args.steps / (ms * 1e-3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8 weights x (bf16-class hi/lo fp8 activations)",
        "data": "synthetic (random-init FP8 experts, Zipf(1.1) top-8 per token)",
        "config": {"workload": "prefill-gather", "tokens": T, "layers": args.layers,
                   "cache_slots_per_layer": cap, "parallelism": f"replicas{world}",
                   "l2": "inputs > L2",
                   "prefetch": ("none: each layer's union gathered after its router"
                                if pf is None or not pf._piped else
                                "every expert of the next layer gathered during this layer's "
                                "GEMM (side stream, two full-layer buffers)")},
        "experts_fetched_per_chunk": fetched, "experts_borrowed_per_chunk": borrowed,
        "gather_gbs": fetch_gbs, "host_link_peak_gbs": peak["gbs"],
        "roofline": {"bound": "host_link", "kernel": "gather_kernel (fetch of the union's misses)",
                     "achieved": fetch_gbs, "peak": peak["gbs"], "unit": "GB/s",
                     "frac": fetch_gbs / peak["gbs"], "traffic": None},
        "moe_ms_per_chunk": layer_ms, "moe_tflops": flops / (layer_ms * 1e-3) / 1e12,
        "clocks": clk.summary(),
        # per layer: router, plan (union path only), gather, and the expert call's launches
        "gpu_launches": args.steps * args.layers * (9 if pf is None or not pf._piped else 8),
    }


# ---------------------------------------------------------------- layer

METRIC_LAYER = "single MoE layer tok/s (T=16, 256 resident FP8 experts, top-8)"


def run_layer(args, rank, world, local):
    """one MoE layer -- router + FP8 expert GEMMs -- over 16 decode
    tokens (hidden 2048, 256 experts resident in HBM, intermediate 512,
    N(0,0.02) weights quantised per 128x128 block, router N(0,0.02), x N(0,1),
    seed 0).  One step = one layer call, graph-replayed; each step routes a
    different 16-token batch (64 prepared batches), so the ~100 distinct
    experts a step reads (~320 MB) come from HBM, not L2.  Parity against the
    oracle (ids bit-exact, hidden rel <= 1e-2) is checked on batch 0; the CPU
    restatement (oracle router + dequantise-then-matmul) is timed on the host
    cores beside it."""
    from drama3_offloading_b200 import benchutil, moe, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T, E, NB = 16, 256, 64
    ex = synth.make_experts(E, seed=0, device="cuda", chunk=32)
    g = torch.Generator().manual_seed(0)
    gate_c = (torch.randn(E, 2048, generator=g) * 0.02).to(torch.bfloat16)
    xs_c = [torch.randn(T, 2048, generator=g).to(torch.bfloat16) for _ in range(NB)]
    gate = gate_c.to(dev)
    xs = torch.stack(xs_c).to(dev)                       # [NB, T, H]
    ids = torch.empty(T, 8, dtype=torch.int32, device=dev)
    wts = torch.empty(T, 8, dtype=torch.float32, device=dev)
    out = torch.empty(T, 2048, dtype=torch.bfloat16, device=dev)
    sel = torch.zeros(1, dtype=torch.int64, device=dev)
    xcur = torch.empty(T, 2048, dtype=torch.bfloat16, device=dev)

    def layer(x):
        moe.router_topk(x, gate, 8, out_ids=ids, out_w=wts)
        moe.fp8_moe_forward(x, ids, wts, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv, out=out)

    def step():
        xcur.copy_(xs.index_select(0, sel)[0])
        sel.add_(1).remainder_(NB)
        layer(xcur)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step()
    for _ in range(max(3, args.warmup)):
        gr.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            gr.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / args.steps
    # distinct experts per batch -> algorithmic HBM bytes of the expert GEMMs
    distinct = []
    for i in range(NB):
        moe.router_topk(xs[i], gate, 8, out_ids=ids, out_w=wts)
        distinct.append(int(torch.unique(ids).numel()))
    alg_bytes = float(np.mean(distinct)) * EXPERT_BYTES + E * 2048 * 2
    # the moe call alone, for the roofline of the expert GEMMs
    evs = []
    for i in range(NB):
        moe.router_topk(xs[i], gate, 8, out_ids=ids, out_w=wts)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        moe.fp8_moe_forward(xs[i], ids, wts, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv, out=out)
        e1.record()
        evs.append((e0, e1, distinct[i]))
    torch.cuda.synchronize(dev)
    moe_ms = float(np.mean([x.elapsed_time(y) for x, y, _ in evs[4:]]))
    moe_gbs = float(np.mean([d * EXPERT_BYTES / (x.elapsed_time(y) * 1e-3) / 1e9
                             for x, y, d in evs[4:]]))
    # e2e through the public API with host buffers: x pinned host -> device,
    # router + experts, out -> pinned host, every step
    hx = xs_c[0].pin_memory()
    ho = torch.empty(T, 2048, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(T, 2048, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        xd.copy_(hx, non_blocking=True); layer(xd); ho.copy_(out, non_blocking=True)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        xd.copy_(hx, non_blocking=True)
        layer(xd)
        ho.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    # parity on batch 0 and the CPU restatement beside it
    import oracle
    layer(xs[0])
    torch.cuda.synchronize(dev)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu_ex = ex.to("cpu")
    t0 = time.perf_counter()
    rid, rw, _, _ = oracle.router_topk(xs_c[0], gate_c, 8)
    ref = oracle.moe_forward(xs_c[0], rid, rw, cpu_ex.w13_weight, cpu_ex.w13_scale_inv,
                             cpu_ex.w2_weight, cpu_ex.w2_scale_inv)
    cpu_s = time.perf_counter() - t0
    ids_exact = bool(np.array_equal(ids.cpu().numpy(), rid.numpy()))
    rel = float((out.float().cpu() - ref).abs().max() / ref.abs().max())
    peak = measured_peaks()
    return {
        "metric": METRIC_LAYER, "value": T / (ms * 1e-3), "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8 weights x (bf16-class hi/lo fp8 activations)",
        "data": "synthetic (configs[0]: N(0,0.02) FP8 experts, bf16 router, N(0,1) tokens, seed 0)",
        "config": {"workload": "single-moe-layer", "tokens": T, "experts": E, "hidden": 2048,
                   "intermediate": 512, "topk": 8, "parallelism": "single",
                   "l2": "inputs > L2 (805 MB of experts, a new 16-token batch each step)"},
        "layer_us": ms * 1e3, "moe_us": moe_ms * 1e3,
        "distinct_experts_per_step": float(np.mean(distinct)),
        "roofline": {"bound": "hbm", "kernel": "d3_moe_fp8_forward (expert GEMMs)",
                     "achieved": moe_gbs, "peak": peak["hbm_gbs"], "unit": "GB/s",
                     "frac": moe_gbs / peak["hbm_gbs"], "traffic": None,
                     "bytes": "distinct experts x 3,146,496 B",
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak['source']})"},
        "layer_roofline_frac": alg_bytes / (peak["hbm_gbs"] * 1e9) / (ms * 1e-3),
        "parity": {"ids_bit_exact": ids_exact, "rel_err": rel, "tolerance": 1e-2},
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": T * 2048 * 2, "d2h_bytes_per_step": T * 2048 * 2},
        "cpu_baseline": {"value": T / cpu_s, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "batch 0 (16 tokens): oracle router + dequantise-then-matmul "
                                   "fp32 experts, torch on all host threads"},
        "clocks": clk.summary(), "gpu_launches": args.steps * 7,
    }


# ---------------------------------------------------------------- ep

def run_ep(args, rank, world, local):
    """Fully resident expert-parallel decode: 256 experts sharded 256/N per
    GPU, global batch 64 split over the ranks, uniform-random top-8 routing,
    dispatch/combine over NVLink peer stores (or NCCL all-to-all with
    --ep-exchange nccl), 40 layers per step in one CUDA graph."""
    from drama3_offloading_b200 import benchutil, moe
    from drama3_offloading_b200.ep import ExpertParallelMoE, synth_expert_bytes
    from drama3_offloading_b200.trace import uniform_trace

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    trace = uniform_trace(steps=256, tokens=args.global_batch, layers=args.layers)
    m = ExpertParallelMoE(layers=args.layers, global_batch=args.global_batch, rank=rank,
                          world=world, group=local_group(world), device=dev, trace=trace,
                          exchange=args.ep_exchange)
    g = m.capture()
    m.step_idx.zero_()
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    ms = benchutil.max_over_ranks(a.elapsed_time(b), world, dev)
    # the NVLink exchange, timed in one eager step: CUDA events around every
    # layer's dispatch and combine (the combine's wait for the slowest
    # serving rank included); max over ranks
    dispatch_us = combine_us = None
    if m.p2p is not None:
        xe = []
        m.step(xchg_events=xe)
        torch.cuda.synchronize(dev)
        dispatch_us = benchutil.max_over_ranks(
            float(np.mean([d0.elapsed_time(d1) for d0, d1, _, _ in xe])) * 1e3, world, dev)
        combine_us = benchutil.max_over_ranks(
            float(np.mean([c0.elapsed_time(c1) for _, _, c0, c1 in xe])) * 1e3, world, dev)
    # the expert call per rank, timed as it runs in the step -- replayed from a
    # CUDA graph with CUDA events -- on the rows this rank received last, for
    # each layer's weights; bytes = the distinct local experts in those rows
    eb = synth_expert_bytes(2048, 512)
    per_layer_us, per_layer_bytes = [], []
    reps = 10
    # with the NVLink exchange the step runs the folded call
    # (d3_moe_fp8_forward_p2p): time that call, on a local stand-in of the
    # link (dispatch flags already at the epoch, every source's return rows a
    # local scratch), so the replays touch no other rank
    if m.p2p is not None:
        import ctypes
        n = world * m.cap
        lk_flags = torch.ones(world, dtype=torch.int64, device=dev)
        lk_epoch = torch.ones(1, dtype=torch.int64, device=dev)
        lk_ret = torch.empty(n, m.H, dtype=torch.bfloat16, device=dev)
        lk_fr = torch.zeros(world, dtype=torch.int64, device=dev)
        lk_ctr = torch.zeros(1, dtype=torch.int32, device=dev)
        lk_ret_p = (ctypes.c_void_p * world)(*([lk_ret.data_ptr()] * world))
        lk_fr_p = (ctypes.c_void_p * world)(*([lk_fr.data_ptr()] * world))
    for l in range(args.layers):
        wl = m.w[l]
        if m.exchange == "none":
            cur = m.trace_dev.index_select(0, m.step_idx)[0][l]
            xin, ids_in, w_in = m.h, cur, m.wts
        else:
            bufs = m.p2p if m.p2p is not None else m
            xin, ids_in, w_in = bufs.recv_x, bufs.recv_eid.view(-1, 1), m.ones
        if m.p2p is not None:
            fn = lambda: moe.fp8_moe_forward_p2p(
                xin, ids_in, w_in, wl.w13_weight, wl.w13_scale_inv, wl.w2_weight,
                wl.w2_scale_inv, wait_flags=lk_flags, epoch=lk_epoch, n_ranks=world, rank=rank,
                cap=m.cap, peer_ret=lk_ret_p, peer_flag_r=lk_fr_p, counter=lk_ctr, wait_code=31,
                budget_ns=m.WAIT_BUDGET_NS)
        else:
            fn = lambda: moe.fp8_moe_forward(xin, ids_in, w_in, wl.w13_weight, wl.w13_scale_inv,
                                             wl.w2_weight, wl.w2_scale_inv, out=m.y if
                                             m.exchange != "none" else None)
        s_ = torch.cuda.Stream(device=dev)
        s_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_):
            fn()
        torch.cuda.current_stream().wait_stream(s_)
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg):
            for _ in range(reps):
                fn()
        gg.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gg.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        per_layer_us.append(e0.elapsed_time(e1) * 1e3 / reps)
        used = ids_in.reshape(-1).cpu().numpy()
        used = used[(used >= 0) & (used < m.epr)] if m.exchange != "none" else used
        per_layer_bytes.append(len(np.unique(used)) * eb)
        del gg
    gemm_us = float(np.mean(per_layer_us))
    gemm_gbs = float(np.sum(per_layer_bytes)) / (float(np.sum(per_layer_us)) * 1e-6) / 1e9
    hbm = measured_peaks()["hbm_gbs"]
    gbs_all = [0.0] * world
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([gemm_gbs], device=dev, dtype=torch.float64)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        gbs_all = [float(x.item()) for x in out]
    else:
        gbs_all = [gemm_gbs]
    overflow = int(m.overflow.item())
    moe.check_errors(dev)   # a bounded exchange wait that ran out would show here
    g = None
    m.close()
    value = args.global_batch * args.steps / (ms * 1e-3)
    exch = {"p2p": "NVLink peer stores + epoch flags (CUDA IPC), static capacity",
            "nccl": "NCCL all-to-all, static capacity", "none": "none"}[m.exchange]
    per_layer = {"p2p": 8, "nccl": 9, "none": 6}[m.exchange]
    return {
        "metric": "resident expert-parallel decode tok/s (40L, batch 64, 256 experts / N GPUs)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8 weights x (bf16-class hi/lo fp8 activations)",
        "data": "synthetic (random-init FP8 experts, uniform-random top-8 routing)",
        "config": {"workload": "ep-resident-decode", "layers": args.layers, "experts": 256,
                   "experts_per_gpu": m.epr, "global_batch": args.global_batch, "topk": 8,
                   "parallelism": f"ep{world}", "exchange": exch,
                   "l2": f"inputs > L2 ({args.layers * m.epr * eb / 2**30:.1f} GiB resident "
                         f"experts per GPU)"},
        "expert_call_us": gemm_us,
        "roofline": {"bound": "hbm", "kernel": "expert GEMMs (d3_moe_fp8_forward, per rank)",
                     "achieved": gemm_gbs, "peak": hbm, "unit": "GB/s", "frac": gemm_gbs / hbm,
                     "traffic": None, "per_rank_gbs": gbs_all,
                     "bytes": "distinct local experts x 3,146,496 B per layer",
                     "timing": "the rank's expert call as the step runs it (with the NVLink "
                               "exchange: the folded call on a local stand-in of the link) "
                               "replayed from a CUDA graph (10 calls) per layer on its last "
                               "received rows, CUDA events",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "overflow_pairs": overflow, "clocks": clk.summary(),
        "gpu_launches": args.steps * args.layers * per_layer,
        "exchange_dispatch_us": dispatch_us, "exchange_combine_us": combine_us,
        "limiter": ep_limiter(ms / args.steps / args.layers * 1e3, gemm_us, dispatch_us,
                              combine_us),
    }


def ep_limiter(layer_us, expert_us, dispatch_us, combine_us) -> str:
    """Which part of an expert-parallel layer step the time goes to."""
    parts = {"expert call (route + GEMMs + act + combine-return)": expert_us}
    if dispatch_us is not None:
        parts["NVLink dispatch"] = dispatch_us
        parts["combine incl. wait for the slowest rank"] = combine_us
    top = max(parts, key=parts.get)
    return (f"{top}: {parts[top]:.1f} of {layer_us:.1f} us per layer "
            f"({', '.join(f'{k} {v:.1f}' for k, v in parts.items())})")


# ---------------------------------------------------------------- ep-rank (configs[4], one rank)

def run_ep_rank(args, rank, world, local):
    """One rank's expert call at the N-GPU expert-parallel shape, on one GPU:
    the rank's 256/N local experts per layer and its received rows (N sources
    x cap = (64/N)*8 rows, one routed pair each, uniform top-8 routing of the
    64-token batch, the rest -1) -- exactly what the expert call of an N-GPU
    step sees -- through the folded NVLink call (d3_moe_fp8_forward_p2p) on a
    local stand-in of the link (dispatch flags already at the epoch, return
    rows local), replayed from a CUDA graph.  Isolates the per-rank expert
    GEMMs from the exchange, for the roofline at every N on one GPU."""
    import ctypes
    from drama3_offloading_b200 import benchutil, moe, synth
    from drama3_offloading_b200.ep import synth_expert_bytes

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N = args.ep_ranks
    epr, T_local = 256 // N, args.global_batch // N
    cap = T_local * 8
    rows = N * cap
    layers = args.layers
    rng = np.random.default_rng(3)
    eb = synth_expert_bytes(2048, 512)
    ws = [synth.make_experts(epr, seed=l, device=dev, chunk=16) for l in range(layers)]
    x = torch.randn(rows, 2048, device=dev).to(torch.bfloat16)
    ids_l, nd = [], []
    for l in range(layers):
        ids = np.full(rows, -1, np.int32)
        for s_ in range(N):
            toks = np.stack([rng.permutation(256)[:8] for _ in range(T_local)])
            mine = toks[toks // epr == 0] % epr
            ids[s_ * cap: s_ * cap + len(mine)] = mine
        ids_l.append(torch.from_numpy(ids).to(dev).view(-1, 1))
        nd.append(len(np.unique(ids[ids >= 0])))
    ones = torch.ones(rows, 1, device=dev)
    ret = torch.zeros(rows, 2048, dtype=torch.bfloat16, device=dev)
    flag_r = torch.zeros(N, dtype=torch.int64, device=dev)
    flag_d = torch.ones(N, dtype=torch.int64, device=dev)
    epoch = torch.ones(1, dtype=torch.int64, device=dev)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    peer_ret = (ctypes.c_void_p * N)(*([ret.data_ptr()] * N))
    peer_fr = (ctypes.c_void_p * N)(*([flag_r.data_ptr()] * N))

    def call(l):
        w = ws[l]
        moe.fp8_moe_forward_p2p(x, ids_l[l], ones, w.w13_weight, w.w13_scale_inv, w.w2_weight,
                                w.w2_scale_inv, wait_flags=flag_d, epoch=epoch, n_ranks=N,
                                rank=0, cap=cap, peer_ret=peer_ret, peer_flag_r=peer_fr,
                                counter=ctr, wait_code=31, budget_ns=2_000_000_000)

    def step():
        for l in range(layers):
            call(l)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with benchutil.ClockSampler(local) as clk:
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("timed")
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    moe.check_errors(dev)
    us = a.elapsed_time(b) * 1e3 / (args.steps * layers)
    byt = float(np.mean(nd)) * eb
    hbm = measured_peaks()["hbm_gbs"]
    gbs = byt / (us * 1e-6) / 1e9
    return {
        "metric": "per-rank expert call us (folded NVLink call, one rank of the N-GPU "
                  "expert-parallel step, emulated on one GPU)",
        "value": us, "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": us * layers / 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8 weights x (bf16-class hi/lo fp8 activations)",
        "data": "synthetic (random-init FP8 experts, uniform-random top-8 routing)",
        "config": {"workload": "ep-rank", "ranks_emulated": N, "experts_per_rank": epr,
                   "received_rows": rows, "valid_pairs_per_layer": int(np.mean(
                       [int((i >= 0).sum()) for i in ids_l])), "layers": layers,
                   "fused_one_launch": os.environ.get("D3_MOE_FUSED", "0") == "1",
                   "l2": f"inputs > L2 ({layers * epr * eb / 2**30:.1f} GiB of experts)"},
        "distinct_experts_per_layer": float(np.mean(nd)),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "traffic": None,
                     "bytes": "distinct local experts x 3,146,496 B per layer"},
        "clocks": clk.summary(), "gpu_launches": args.steps * layers * 5,
    }


# ---------------------------------------------------------------- main

def reference_arm(args, rank):
    """--impl reference: the reference's CPU path (oracle port) on this box's
    host cores, rank 0 only, one bounded sample per step."""
    if rank != 0:
        return
    from drama3_offloading_b200.trace import zipf_trace
    trace = zipf_trace(steps=4096, layers=args.layers)
    if args.workload == "fetch":
        cap = max(1, args.slots // args.layers)
        per = max(0.05, args.cpu_sample_s / max(1, args.steps + args.warmup))
        res = [cpu_fetch_baseline(trace, cap, per) for _ in range(args.warmup + args.steps)]
        v = float(np.mean([r["value"] for r in res[args.warmup:]]))
        unit, metric, dtype, r = "GB/s", METRIC_FETCH, "u8", res[-1]
        cfg = {"workload": "fetch", "layers": args.layers, "slots": args.slots}
    else:
        cap = max(1, int(args.cache_gib * (1 << 30)) // (args.layers * EXPERT_BYTES))
        nl = max(1, min(args.layers, args.cpu_layers))
        cpu = CpuDecodeSample(nl, trace, cap)
        for _ in range(args.warmup):
            cpu.token()
        ts = [cpu.token() for _ in range(args.steps)]
        v = 1.0 / (float(np.mean(ts)) / nl * args.layers)
        unit, metric = "tok/s", METRIC_DECODE
        dtype = "fp8 weights x bf16 activations (fp32 accumulate), bf16 dense"
        r = {"cores": cpu.threads, "kind": "port",
             "sample": f"each step: one token through {nl} of {args.layers} layers (time x "
                       f"{args.layers}/{nl}); torch bf16 dense GEMVs + KV-context attention + "
                       f"oracle router/LRU + expert memcpy + dequantised fp32 expert matmuls "
                       f"+ shared expert"}
        cfg = decode_config(args)
    line = {"impl": "reference", "metric": metric, "value": v, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": v, "unit": unit, "cores": r["cores"], "kind": r["kind"],
                             "sample": r["sample"]},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local = init_dist(args)
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if args.workload in ("ep", "ep-rank", "prefill", "layer"):
        run = {"ep": run_ep, "ep-rank": run_ep_rank, "prefill": run_prefill,
               "layer": run_layer}[args.workload]
        r = run(args, rank, world, local)
        if rank == 0:
            print(json.dumps(r), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    ep_rec = None
    if args.workload == "fetch":
        r = run_fetch(args, rank, world, local)
    else:
        r = run_decode(args, rank, world, local)
        if not args.no_ep:
            # the resident expert-parallel configuration at the same
            # N, after the decode stack is gone: a sub-record of the same line
            import gc
            gc.collect()
            torch.cuda.empty_cache()
            ep_rec = run_ep(args, rank, world, local)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            if args.workload == "fetch":
                cpu = cpu_fetch_baseline(r["trace"], r["capacity"], args.cpu_sample_s)
            else:
                cpu = cpu_decode_baseline(r["trace"], r["capacity"], args.layers, args.cpu_layers,
                                          args.cpu_sample_s)
        peak = r["peak"]["gbs"]
        if args.workload == "fetch":
            line = {
                "metric": METRIC_FETCH, "value": r["value"], "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"] / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
                "data": "synthetic (random N(0,0.02) FP8 weights, seeded Zipf(1.1) trace)",
                "config": {"workload": "expert-fetch", "layers": args.layers, "experts": 256,
                           "slots": args.slots, "slots_per_layer": r["capacity"],
                           "policy": args.policy, "l2": "inputs (30 GiB host store) > L2",
                           "parallelism": f"replicas{world}"},
                "hit_rate": r["hit_rate"], "misses_per_step": r["misses_per_step"],
                "host_link_peak_gbs": peak,
                "roofline": {"bound": "host_link", "achieved": r["gbs_rank"], "peak": peak,
                             "unit": "GB/s", "frac": r["gbs_rank"] / peak, "traffic": None},
                "clocks": r["clk"], "gpu_launches": r["launches"],
            }
        else:
            tokb = r["value"] / world
            misses_per_launch = r["misses"] / args.layers
            traffic = (FETCH_PCIE_BYTES_PER_EXPERT * misses_per_launch
                       if FETCH_PCIE_BYTES_PER_EXPERT else None)
            line = {
                "metric": METRIC_DECODE, "value": r["value"], "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"] / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "fp8 weights x bf16 activations (fp32 accumulate), bf16 dense",
                "data": "synthetic (random-init Drama-3 shapes, seeded Zipf(1.1) routing trace)",
                "config": decode_config(args, r["capacity"]),
                "hits_per_token": r["hits"], "misses_per_token": r["misses"],
                "hit_rate": r["hits"] / max(1e-9, r["hits"] + r["misses"]),
                "fetch_gbs": r["fetch_gbs"], "host_link_peak_gbs": peak,
                "fetch_frac_of_host_peak": r["fetch_gbs"] / peak,
                "fetch_window": "the timed window again from the same cache state, eager, "
                                "CUDA events around every layer's fetch launch",
                "token_roofline_ms": r["roof_ms"],
                "token_roofline_frac": r["roof_ms"] / (1e3 / tokb),
                "roofline": {"bound": "host_link",
                             "kernel": ("fetch_gemv13_kernel: the fetch with the gate/up "
                                        "products overlapped (event-timed launch)"
                                        if not args.no_overlap
                                        else "fetch_layer_kernel (+allocator)"),
                             "achieved": r["fetch_gbs"], "peak": peak, "unit": "GB/s",
                             "frac": r["fetch_gbs"] / peak, "traffic": traffic,
                             "traffic_unit": "PCIe read bytes per launch (ncu "
                                             "pcie__read_bytes.sum per fetched expert x "
                                             "experts fetched per launch in this window)",
                             "algorithmic_bytes": misses_per_launch * EXPERT_BYTES,
                             "peak_source": "measured pinned copy-engine H2D, this run"},
                "e2e": {"value": r["e2e"], "unit": "tok/s", "h2d_bytes_per_step": 2 * 2048,
                        "d2h_bytes_per_step": 2 * 2048,
                        "window": f"the timed window from the same state ({r['e2e_steps']} "
                                  "steps), host sync every token"},
                "clocks": r["clk"], "gpu_launches": r["launches"],
                "host_store": r["host_store"],
            }
        if ep_rec is not None:
            line["ep"] = {k: ep_rec[k] for k in (
                "metric", "value", "unit", "n_gpus", "ms_per_step", "expert_call_us",
                "exchange_dispatch_us", "exchange_combine_us", "limiter", "overflow_pairs",
                "gpu_launches", "config")}
            line["ep"]["roofline"] = {k: ep_rec["roofline"][k] for k in (
                "bound", "achieved", "peak", "unit", "frac", "per_rank_gbs", "bytes")}
        line["cpu_baseline"] = None if cpu is None else {
            k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
