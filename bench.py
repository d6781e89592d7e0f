"""Benchmark of the routed-MoE expert-offload hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W] [--impl ours|reference]

Workloads:

* ``fetch``  -- configs[1], the expert-fetch microbenchmark: 40 layers x 256
  experts of FP8 weights + scales (30 GiB) in pinned host memory, per-layer
  device caches totalling 2048 slots (51 per layer), the synthetic Zipf(1.1)
  routing trace (top-8 per layer), one decode step = 40 x (allocator + fused
  fetch) replayed from a CUDA graph.  Metric: fetch GB/s vs the measured
  host-link (pinned copy-engine) peak.

A step is one decode step over all 40 layers.  Inputs (the 30 GiB host store)
are far larger than L2.  Multi-GPU runs are replicas (each rank its own store
and link; "scaling": "weak").
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("fetch",), default="fetch")
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--slots", type=int, default=2048, help="device cache slots over all layers")
    ap.add_argument("--policy", choices=("lru", "lfu"), default="lru")
    ap.add_argument("--fetch-ctas", type=int, default=0)
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def init_dist(args):
    from drama3_offloading_b200.benchutil import dist_env
    rank, world, local = dist_env()
    if world > 1:
        import torch.distributed as dist
        if args.impl == "ours" or torch.cuda.is_available():
            torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    return rank, world, local


# ---------------------------------------------------------------- CPU legs

def cpu_fetch_baseline(trace: np.ndarray, capacity: int, policy: str, sample_s: float) -> dict:
    """The oracle's allocator plus a memcpy of every missed expert (host store
    -> host cache), timed on this box's cores over a bounded sample of the
    same trace.  One thread (the reference's allocator and fetch are serial)."""
    import oracle
    layers = trace.shape[1]
    store = np.random.default_rng(0).integers(0, 255, size=(16, EXPERT_BYTES), dtype=np.uint8)
    cache = np.zeros((capacity, EXPERT_BYTES), dtype=np.uint8)
    tabs = [oracle.init_tables(256, capacity) for _ in range(layers)]
    res = oracle.resolve_lfu if policy == "lfu" else oracle.resolve
    t0 = time.perf_counter()
    steps = misses = 0
    while time.perf_counter() - t0 < sample_s and steps < trace.shape[0]:
        for l in range(layers):
            _, fs, fe, n = res(tabs[l], trace[steps, l])
            for j in range(n):
                cache[fs[j]] = store[int(fe[j]) % 16]
            misses += n
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": misses * EXPERT_BYTES / dt / 1e9, "unit": "GB/s", "cores": 1,
            "kind": "port", "steps": steps, "seconds": dt,
            "sample": f"first {steps} steps x {layers} layers of the Zipf trace, LRU oracle + "
                      f"memcpy of each missed 3,146,496-B expert (host->host)"}


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
                             policy=args.policy, fill="random")
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
    torch.cuda.synchronize(dev)
    # capture one step (capture executes nothing), then restart the trace and
    # the caches cold in place so the replays start from the init state
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
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.synchronize(dev)
    benchutil.barrier(world, dev)
    ms = a.elapsed_time(b)
    c1 = store.counters()
    misses = c1["misses"] - c0["misses"]
    hits = c1["hits"] - c0["hits"]
    fetched = c1["bytes_fetched"] - c0["bytes_fetched"]
    ms_max = benchutil.max_over_ranks(ms, world, dev)
    gbs_rank = fetched / (ms * 1e-3) / 1e9
    total_bytes = benchutil.sum_over_ranks(fetched, world, dev)
    value = total_bytes / (ms_max * 1e-3) / 1e9
    return {
        "value": value, "ms": ms_max, "gbs_rank": gbs_rank, "peak": peak, "clk": clk.summary(),
        "hit_rate": hits / max(1, hits + misses), "misses_per_step": misses / args.steps,
        "capacity": capacity, "setup_s": store.setup_s, "trace": trace,
        "launches": args.steps * args.layers * 2,
    }


def main():
    args = parse()
    rank, world, local = init_dist(args)
    if args.impl == "reference":
        if rank != 0:
            return
        from drama3_offloading_b200.trace import zipf_trace
        trace = zipf_trace(steps=4096, layers=args.layers)
        capacity = max(1, args.slots // args.layers)
        res = []
        for _ in range(args.warmup + args.steps):
            res.append(cpu_fetch_baseline(trace, capacity, args.policy,
                                          args.cpu_sample_s / max(1, args.steps)))
        r = res[-1]
        v = float(np.mean([x["value"] for x in res[args.warmup:]]))
        line = {"impl": "reference", "metric": "expert-fetch GB/s (40L, 2048-slot cache, Zipf(1.1))",
                "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "u8", "data": "synthetic",
                "config": {"workload": "fetch", "layers": args.layers, "slots": args.slots},
                "cpu_baseline": {k: r[k] for k in ("unit", "cores", "kind", "sample")} | {"value": v},
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    r = run_fetch(args, rank, world, local)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_fetch_baseline(r["trace"], r["capacity"], args.policy, args.cpu_sample_s)
        peak = r["peak"]["gbs"]
        line = {
            "metric": "expert-fetch GB/s (40L x 256 experts pinned, 2048-slot cache, Zipf(1.1), graph)",
            "value": r["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms"] / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (random N(0,0.02) FP8 weights, seeded Zipf(1.1) trace)",
            "config": {"workload": "fetch", "layers": args.layers, "experts": 256,
                       "slots": args.slots, "slots_per_layer": r["capacity"],
                       "policy": args.policy, "l2": "inputs (30 GiB host store) > L2",
                       "parallelism": f"replicas{world}"},
            "hit_rate": r["hit_rate"], "misses_per_step": r["misses_per_step"],
            "host_link_peak_gbs": peak,
            "roofline": {"bound": "host_link", "achieved": r["gbs_rank"], "peak": peak,
                         "unit": "GB/s", "frac": r["gbs_rank"] / peak, "traffic": None},
            "clocks": r["clk"], "gpu_launches": r["launches"],
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in (
                "value", "unit", "cores", "kind", "sample")},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
