"""A 40-layer Drama-3-shaped expert store in page-locked host memory with
per-layer device caches -- the offloaded configuration the reference runs in
production (bin/offload.py:111-134 materialize_offloaded, :664-699
pin_experts; bin/devcache.py:280-301 install_dev_cache).

Weights are random-init (no checkpoint): N(0, 0.02) quantised per 128x128
block, generated on the GPU a few experts at a time and copied into the host
store.  The store is one shared, page-locked allocation per machine
(``hoststore.SharedHostStore``), one copy per NUMA node holding the ranks'
GPUs: local rank 0 fills its copy, the owners of the other nodes' copies copy
it, every local rank maps its node's copy and keeps its own device cache.
"""
from __future__ import annotations

import time

import torch

from . import devcache, synth
from .hoststore import SharedHostStore, gpu_numa_node, layer_bytes

GiB = 1 << 30


def fill_layer(host: synth.HostExperts, seed: int, device, fill: str = "random",
               gen_chunk: int = 32) -> None:
    E = host.num_experts
    H = host.w13_weight.shape[2]
    I = host.w2_weight.shape[2]
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
        host.w13_weight.view(torch.uint8).zero_()
        host.w2_weight.view(torch.uint8).zero_()
        host.w13_scale_inv.fill_(1.0)
        host.w2_scale_inv.fill_(1.0)
    else:
        raise ValueError(fill)


class OffloadedExperts:
    """``layers`` host expert stores (one shared page-locked allocation), each
    with its own device cache on ``device``.

    ``group``/``local_rank``: the ranks of this machine share the store (one
    copy per NUMA node of their GPUs, ``per_node``); local rank 0 fills it."""

    def __init__(self, layers: int = 40, experts: int = 256, hidden: int = 2048,
                 inter: int = 512, capacity: int = 51, device="cuda", seed: int = 0,
                 policy: str = "lru", fill: str = "random", group=None, local_rank: int = 0,
                 per_node: bool = True):
        import torch.distributed as dist
        self.device = torch.device(device)
        self.H, self.I, self.E = hidden, inter, experts
        t0 = time.perf_counter()
        self.host = SharedHostStore(layers * layer_bytes(experts, hidden, inter), local_rank,
                                    group, node=gpu_numa_node(self.device), per_node=per_node)
        self.layers = []
        for l in range(layers):
            ex = synth.HostExperts(
                experts,
                self.host.take((experts, 2 * inter, hidden), torch.float8_e4m3fn),
                self.host.take((experts, hidden, inter), torch.float8_e4m3fn),
                self.host.take((experts, 2 * inter // 128, hidden // 128), torch.float32),
                self.host.take((experts, hidden // 128, inter // 128), torch.float32))
            self.layers.append(ex)
        multi = group is not None and dist.is_initialized() and dist.get_world_size(group) > 1
        # local rank 0 page-locks and fills its copy first; the owners of the
        # other nodes' copies copy it and page-lock theirs; the other ranks
        # page-lock their node's filled copy last
        if self.host.primary:
            self.host.register()
            for l, ex in enumerate(self.layers):
                fill_layer(ex, seed + l, self.device, fill)
        torch.cuda.synchronize(self.device)
        if multi:
            dist.barrier(group=group, device_ids=[self.device.index])
        if self.host.copies > 1:
            if self.host.owner and not self.host.primary:
                self.host.copy_from_primary()
                self.host.register()
            if multi:
                dist.barrier(group=group, device_ids=[self.device.index])
        if not self.host.owner:
            self.host.register()
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
