"""40-layer Drama-3-shaped MoE decode stack with experts offloaded to pinned host
memory -- the production configuration of the reference (device cache + fetch
kernel + CUDA graphs, bin/narrate.py:573-650, notes/12-full-run.md:6-10),
random-initialised at the real shapes.

Per layer and decode token (batch 1):

1. dense stand-in: ``h += down(silu(up(h)))`` with bf16 weights sized so the
   40 layers read 6.9 GiB per token together with the shared experts -- the
   non-routed (attention / GDN / shared-expert / projection) weight traffic
   of Drama-3 (notes/01-static-findings.md:54-55, :80-82).  Plain cuBLAS
   GEMVs: not part of the hot path.
2. router ``d3_router_topk`` on the layer's bf16 gate [256, 2048].
3. ``d3_resolve_fetch_moe`` (default, ``overlap=True``): device slot
   allocator; ONE launch that fetches the missed experts from pinned host
   memory into the layer's device cache on 64 CTAs while the other CTAs run
   the gate/up products of the resident experts and of the layer's gated bf16
   shared expert (resident, 6 MiB), then those of each fetched expert once its
   bytes have landed; then the down projection, accumulated into ``h``.
   (``overlap=False``: ``d3_resolve_fetch``, then ``d3_moe_fp8_forward_shared``
   on the cache slots.)

Drama-3's ten full-attention layers (``layer_types``: every fourth layer,
notes/drama3-config.json; 2 KV heads x 256 dims) also read a 2048-token KV
context per decode token: 4 MiB per such layer, 40 MiB per token.  The stand-in
attends the layer's hidden state (as 2 KV groups x 4 query rows) over a
resident bf16 K/V cache of that size with two batched GEMVs and a softmax
(cuBLAS / torch), so those bytes are read every token too.

Routing: the router runs every layer (its cost is real), but the expert ids
fed to the cache come from the seeded Zipf(1.1) trace so hit rates are those
of skewed real routing rather than of a random-init gate (which routes almost
uniformly).  The router's weights are used for the combine.

The whole token step is captured into one CUDA graph; the trace position is a
device counter, so replays walk the trace.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib, devcache, moe
from .stack import OffloadedExperts

DENSE_GIB = 6.9
KV_CONTEXT = 2048        # cached tokens of every full-attention layer
KV_HEADS, HEAD_DIM = 2, 256


def full_attention_layers(layers: int) -> list:
    """Drama-3's layer_types: layers 3, 7, 11, ... are full attention."""
    return [l for l in range(layers) if l % 4 == 3]


def dense_stand_in_rows(layers: int, hidden: int, inter: int, dense_gib: float) -> int:
    """Rows R of each layer's up [R, H] / down [H, R] bf16 stand-in: the
    layer's share of the dense budget minus its shared expert."""
    shared_bytes = (3 * inter * hidden + hidden) * 2
    per_layer = dense_gib * (1 << 30) / layers - shared_bytes
    return max(128, int(per_layer / (2 * hidden * 2)) // 128 * 128)


def dense_bytes_per_token(layers: int = 40, hidden: int = 2048, inter: int = 512,
                          dense_gib: float = DENSE_GIB, kv_context: int = KV_CONTEXT) -> int:
    """bf16 bytes the non-routed part of one decode token reads: the dense
    stand-in, the shared experts and the full-attention layers' KV context."""
    R = dense_stand_in_rows(layers, hidden, inter, dense_gib)
    shared_bytes = (3 * inter * hidden + hidden) * 2
    kv = len(full_attention_layers(layers)) * 2 * kv_context * KV_HEADS * HEAD_DIM * 2
    return layers * (2 * R * hidden * 2 + shared_bytes) + kv


class DecodeStack:
    def __init__(self, layers: int = 40, experts: int = 256, hidden: int = 2048, inter: int = 512,
                 topk: int = 8, cache_gib: float = 8.0, capacity: int | None = None,
                 dense_gib: float = DENSE_GIB, trace: np.ndarray | None = None, device="cuda",
                 policy: str = "lru", seed: int = 0, fill: str = "random", group=None,
                 local_rank: int = 0, trace_offset: int = 0, overlap: bool = True,
                 kv_context: int = KV_CONTEXT, host_per_node: bool = True,
                 l2_warm_mib: float = 85.0, l2_warm_gate: bool = True):
        self.device = dev = torch.device(device)
        self.overlap = overlap
        # with the overlapped fetch: MiB of the next layer's first dense weight
        # hinted into L2 while this layer's fetch holds the host link
        self.l2_warm_bytes = int(l2_warm_mib * (1 << 20))
        # ... and the next layer's router gate weight with it
        self.l2_warm_gate = l2_warm_gate
        self.L, self.E, self.H, self.I, self.k = layers, experts, hidden, inter, topk
        per_expert = 2 * inter * hidden + hidden * inter + 4 * (2 * inter * hidden + hidden * inter) // (128 * 128)
        self.capacity = capacity or max(1, int(cache_gib * (1 << 30)) // (layers * per_expert))
        self.store = OffloadedExperts(layers, experts, hidden, inter, self.capacity, dev, seed,
                                      policy, fill, group=group, local_rank=local_rank,
                                      per_node=host_per_node)
        self.trace_offset = trace_offset
        g = torch.Generator(device=dev).manual_seed(seed + 7)
        # the shared expert of every layer (bf16 gate/up [2I, H], down [H, I],
        # sigmoid gate [H]), resident; its bytes come out of the dense budget
        self.shared = [((torch.randn(2 * inter, hidden, generator=g, device=dev) * 0.02)
                        .to(torch.bfloat16),
                        (torch.randn(hidden, inter, generator=g, device=dev) * 0.02)
                        .to(torch.bfloat16),
                        (torch.randn(hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16))
                       for _ in range(layers)]
        shared_bytes = (3 * inter * hidden + hidden) * 2
        # dense stand-in: 2 * R * H bf16 per layer
        R = dense_stand_in_rows(layers, hidden, inter, dense_gib)
        self.R = R
        self.up = [torch.randn(R, hidden, generator=g, device=dev, dtype=torch.bfloat16) * (hidden ** -0.5)
                   for _ in range(layers)]
        self.down = [torch.randn(hidden, R, generator=g, device=dev, dtype=torch.bfloat16) * (R ** -0.5 * 0.5)
                     for _ in range(layers)]
        # the full-attention layers' KV context: K and V [KV_HEADS, ctx, HEAD_DIM]
        self.kv_context = kv_context
        self.kv = {}
        if kv_context > 0 and hidden % (KV_HEADS * HEAD_DIM) == 0:
            for l in full_attention_layers(layers):
                k = torch.randn(KV_HEADS, kv_context, HEAD_DIM, generator=g, device=dev) * 0.5
                v = torch.randn(KV_HEADS, kv_context, HEAD_DIM, generator=g, device=dev)
                self.kv[l] = (k.to(torch.bfloat16), v.to(torch.bfloat16))
        self.kv_bytes = sum(k.numel() * 2 + v.numel() * 2 for k, v in self.kv.values())
        self.dense_bytes = (sum(t.numel() * 2 for t in self.up + self.down) +
                            layers * shared_bytes + self.kv_bytes)
        self.gate = [(torch.randn(experts, hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                     for _ in range(layers)]
        self.h = torch.zeros(1, hidden, dtype=torch.bfloat16, device=dev)
        self.ids = torch.empty(1, topk, dtype=torch.int32, device=dev)
        self.wts = torch.empty(1, topk, dtype=torch.float32, device=dev)
        self.moe_out = torch.empty(1, hidden, dtype=torch.bfloat16, device=dev)
        if trace is None:
            from .trace import zipf_trace
            trace = zipf_trace(steps=4096, layers=layers, experts=experts, k=topk)
        self.trace_steps = trace.shape[0]
        self.trace_dev = torch.from_numpy(trace.astype(np.int32)).to(dev)
        self.step_idx = torch.full((1,), trace_offset % self.trace_steps, dtype=torch.int64,
                                   device=dev)
        self.graph = None
        # warm the library (workspaces, smem attributes) outside any capture
        moe.router_topk(self.h, self.gate[0], topk, out_ids=self.ids, out_w=self.wts)

    # ---------------------------------------------------------------- one token
    def _layer(self, l: int, cur_ids: torch.Tensor, events: list | None = None) -> None:
        """h += dense(h); route; resolve + fetch; h += moe(h) -- all in place."""
        h = self.h
        a = torch.nn.functional.silu(h @ self.up[l].t())
        h.addmm_(a, self.down[l].t())
        kv = self.kv.get(l)
        if kv is not None:
            # decode attention over the cached context: q [groups, rows, d]
            k, v = kv
            q = h.view(KV_HEADS, -1, HEAD_DIM)
            p = torch.softmax(torch.bmm(q, k.transpose(1, 2)).float() * HEAD_DIM ** -0.5,
                              dim=-1).to(torch.bfloat16)
            h.add_(torch.bmm(p, v).view(1, -1), alpha=0.25)
        moe.router_topk(h, self.gate[l], self.k, out_ids=self.ids, out_w=self.wts)
        ex = self.store.layers[l]
        if events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if self.overlap:
            # allocator, then fetch + gate/up in one launch, then the down
            # projection (the timing sample brackets the fetch launch alone)
            nxt = (l + 1) % self.L
            warm, caps = [], []
            if self.l2_warm_gate:
                warm.append(self.gate[nxt]); caps.append(None)
            if self.l2_warm_bytes:
                warm.append(self.up[nxt]); caps.append(self.l2_warm_bytes)
            run = lambda stages: devcache.dev_resolve_fetch_moe(
                ex, cur_ids[l], h, self.wts, out=h, accumulate=True, shared=self.shared[l],
                stages=stages, l2_warm=warm or None, l2_warm_bytes=caps or None)
            if events is None:
                run(7)
                return
            run(1)
            e0.record()
            run(2)
            e1.record()
            events.append((e0, e1))
            run(4)
            return
        if events is not None:
            e0.record()
        slots = devcache.dev_resolve_and_fetch(ex, cur_ids[l])
        if events is not None:
            e1.record()
            events.append((e0, e1))
        moe.fp8_moe_forward(h, slots.reshape(1, self.k), self.wts, ex._dc_w13, ex._dc_s13,
                            ex._dc_w2, ex._dc_s2, out=h, accumulate=True,
                            shared=self.shared[l])

    def step(self) -> None:
        """One decode token through all layers (eager; capturable)."""
        cur = self.trace_dev.index_select(0, self.step_idx)[0]
        self.step_idx.add_(1).remainder_(self.trace_steps)
        for l in range(self.L):
            self._layer(l, cur)

    def capture(self) -> torch.cuda.CUDAGraph:
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.step()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.graph = g
        self.reset()
        return g

    _TABLES = ("_dc_slot_of", "_dc_slot_expert", "_dc_stamp", "_dc_step", "_dc_freq",
               "_dc_ins", "_dc_out", "_dc_fslot", "_dc_fexp", "_dc_nmiss", "_dc_counters",
               "_dc_w13", "_dc_w2", "_dc_s13", "_dc_s2")

    def snapshot(self) -> dict:
        """A device copy of everything a replay changes -- every layer's slot
        tables, job table, counters and cache bytes, the hidden state and the
        trace position -- so the same window of tokens can be run again from
        the same state (``restore``)."""
        torch.cuda.synchronize(self.device)
        return {"layers": [[getattr(ex, n).clone() for n in self._TABLES]
                           for ex in self.store.layers],
                "h": self.h.clone(), "step_idx": self.step_idx.clone()}

    def restore(self, snap: dict) -> None:
        """Copy a ``snapshot`` back in place (addresses unchanged, so captured
        graphs stay valid)."""
        for ex, saved in zip(self.store.layers, snap["layers"]):
            for n, t in zip(self._TABLES, saved):
                getattr(ex, n).copy_(t)
        self.h.copy_(snap["h"])
        self.step_idx.copy_(snap["step_idx"])
        torch.cuda.synchronize(self.device)

    def reset(self) -> None:
        """Cold caches, trace at its start, zero hidden state (addresses unchanged)."""
        self.store.reset_caches()
        self.step_idx.fill_(self.trace_offset % self.trace_steps)
        self.h.zero_()
        torch.cuda.synchronize(self.device)

    def sample_fetch_timing(self, steps: int) -> dict:
        """Eager decode steps with CUDA events around every layer's fetch
        (with overlap: the fetch + gate/up launch alone; without: the
        allocator + fetch launch pair): bytes fetched and device time, for the
        fetch kernel's achieved host-link bandwidth."""
        evs = []
        c0 = self.store.counters()
        for _ in range(steps):
            cur = self.trace_dev.index_select(0, self.step_idx)[0]
            self.step_idx.add_(1).remainder_(self.trace_steps)
            for l in range(self.L):
                self._layer(l, cur, evs)
        torch.cuda.synchronize(self.device)
        c1 = self.store.counters()
        ms = sum(a.elapsed_time(b) for a, b in evs)
        return {"bytes": c1["bytes_fetched"] - c0["bytes_fetched"], "ms": ms,
                "launch_pairs": len(evs), "misses": c1["misses"] - c0["misses"]}

    def launches_per_step(self) -> int:
        """Kernels of this library launched per token: router, allocator, fetch,
        and the batch-1 expert path's gate/up and down launches per layer
        (with overlap the fetch and the gate/up products are one launch)."""
        return (4 if self.overlap else 5) * self.L

    def roofline_ms(self, hits: float, misses: float, hbm_gbs: float, host_gbs: float) -> float:
        """t >= dense/HBM + hits*expert/HBM + misses*expert/host per token."""
        eb = devcache.EXPERT_BYTES
        return 1e3 * (self.dense_bytes / (hbm_gbs * 1e9) + hits * eb / (hbm_gbs * 1e9)
                      + misses * eb / (host_gbs * 1e9))
