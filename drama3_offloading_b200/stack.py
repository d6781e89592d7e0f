"""A 40-layer Drama-3-shaped expert store in pinned host memory with per-layer
device caches -- the offloaded configuration the reference runs in production
(bin/offload.py:111-134 materialize_offloaded, :664-699 pin_experts;
bin/devcache.py:280-301 install_dev_cache).

Weights are random-init (no checkpoint): N(0, 0.02) quantised per 128x128
block, generated on the GPU a few experts at a time and copied into
page-locked host buffers (one pinned allocation per layer and buffer, as
pin_experts does; every size is a power of two at the real dims, so the
caching host allocator wastes nothing).
"""
from __future__ import annotations

import time

import torch

from . import devcache, synth

GiB = 1 << 30


def pinned_layer(E: int, H: int, I: int, seed: int, device, fill: str = "random",
                 gen_chunk: int = 32) -> synth.HostExperts:
    host = synth.HostExperts(
        E,
        torch.empty(E, 2 * I, H, dtype=torch.float8_e4m3fn, pin_memory=True),
        torch.empty(E, H, I, dtype=torch.float8_e4m3fn, pin_memory=True),
        torch.empty(E, 2 * I // 128, H // 128, dtype=torch.float32, pin_memory=True),
        torch.empty(E, H // 128, I // 128, dtype=torch.float32, pin_memory=True))
    if fill == "random":
        for lo in range(0, E, gen_chunk):
            hi = min(E, lo + gen_chunk)
            part = synth.make_experts(hi - lo, H, I, seed=seed * 100003 + lo, device=device,
                                      chunk=gen_chunk)
            host.w13_weight[lo:hi].copy_(part.w13_weight)
            host.w2_weight[lo:hi].copy_(part.w2_weight)
            host.w13_scale_inv[lo:hi].copy_(part.w13_scale_inv)
            host.w2_scale_inv[lo:hi].copy_(part.w2_scale_inv)
    elif fill == "zeros":
        for n in ("w13_weight", "w2_weight"):
            getattr(host, n).view(torch.uint8).zero_()
        host.w13_scale_inv.fill_(1.0)
        host.w2_scale_inv.fill_(1.0)
    else:
        raise ValueError(fill)
    return host


class OffloadedExperts:
    """``layers`` pinned host expert stores, each with its own device cache."""

    def __init__(self, layers: int = 40, experts: int = 256, hidden: int = 2048,
                 inter: int = 512, capacity: int = 51, device="cuda", seed: int = 0,
                 policy: str = "lru", fill: str = "random"):
        self.device = torch.device(device)
        self.H, self.I, self.E = hidden, inter, experts
        t0 = time.perf_counter()
        self.layers = [pinned_layer(experts, hidden, inter, seed + l, self.device, fill)
                       for l in range(layers)]
        torch.cuda.synchronize(self.device)
        self.setup_s = time.perf_counter() - t0
        for ex in self.layers:
            devcache.init_dev_cache(ex, self.device, capacity, policy=policy)
        self.capacity = capacity
        self.host_bytes = sum(sum(getattr(ex, n).numel() * getattr(ex, n).element_size()
                                  for n in ("w13_weight", "w2_weight", "w13_scale_inv",
                                            "w2_scale_inv")) for ex in self.layers)

    def reset_caches(self) -> None:
        """Cold caches, same device addresses (captured graphs stay valid)."""
        for ex in self.layers:
            devcache.reset_dev_cache(ex)

    def counters(self) -> dict:
        tot = torch.stack([ex._dc_counters for ex in self.layers]).sum(0).tolist()
        return {"calls": tot[0], "hits": tot[1], "misses": tot[2], "bytes_fetched": tot[3]}
