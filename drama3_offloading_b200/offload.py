"""Prefill (multi-row) MoE over offloaded experts -- drop-in for the hot-path
parts of the reference's ``bin/offload.py``.

* ``offloaded_forward(self, x, topk_ids, topk_weights)`` (bin/offload.py:137-239):
  the distinct routed experts of the batch are gathered into a compact device
  buffer -- cached ones copied read-only from the device cache (the reference's
  HYBRID_GATHER borrow, :195-224: no stamp bump, no insert), the rest fetched
  from pinned host memory -- then the FP8 grouped GEMM runs on the compact set
  with the ids remapped.  Unlike the reference (``torch.unique(ids.cpu())``, a
  host sync per layer, then one ``copy_`` per expert and buffer), the union,
  the remap and the gather are three device launches with static shapes.
* ``ChunkPrefetch`` (no counterpart in the reference): for prefill chunks,
  whose every layer routes to all of its experts, the next layer's experts are
  gathered on a side stream while this layer's expert GEMM runs, so the host
  link never waits for a GEMM; ``install_offload(..., chunk_prefetch=True)``
  puts the installed forward on it.
* ``STATS``, ``HYBRID_GATHER``, ``GATHER_DONE_HOOK``, ``EXPERT_BYTES``,
  ``pin_experts``, ``size_cache_to_free_vram``, ``install_offload`` keep the
  reference's names and meaning (:242-254, :603-704).

Gather counts are kept on the device (``gather_counters(experts)``) rather
than as host-side STATS increments, which would need a sync.

Routing observability (bin/offload.py:40-79, :257-287): ``TRACE``
(``RouterTrace``: ``enabled``, ``add``, ``records``, ``save``,
``first_decode``) and ``enable_census`` / ``CENSUS`` / ``CENSUS_DECODE`` keep
the reference's names, but the ids never leave the device on the hot path:
the census is an int64 [layers, experts] device tensor updated by
``d3_census_add`` and the trace a device ring filled by ``d3_trace_append``.
Both are read (one sync) only when the host asks.  Calls hook them at the top
of ``offloaded_forward``, as the reference does (its device-cache decode path
is not traced either).
"""
from __future__ import annotations

import ctypes
import time

import torch

from . import _lib, moe

EXPERT_BYTES = 3_146_496
HYBRID_GATHER = True
GATHER_DONE_HOOK = None
ACTIVATION_HEADROOM_GIB = 1.5
STATS = {"experts_copied": 0, "bytes_copied": 0, "hits": 0, "misses": 0,
         "gather_hits": 0, "gather_misses": 0}

_BUF: dict = {}
# install_offload(..., chunk_prefetch=True): the offloaded layers in model order
# and their shared ChunkPrefetch (made on the first multi-row call)
_CHAIN: dict = {"layers": [], "pf": None}


# ---------------------------------------------------------------- trace

class RouterTrace:
    """Every (layer, routed row) -> its top-k expert ids, in a device ring.

    ``add`` launches one kernel (no host sync, graph-capturable); ``records``
    reads the ring back and groups rows into the reference's per-call records
    ``{"phase": "decode"|"prefill", "layer": l, "ids": [[...], ...]}`` (a call
    of one row is decode).  ``capacity`` rows are kept; older rows are
    overwritten and ``dropped`` counts them."""

    def __init__(self, capacity: int = 1 << 16) -> None:
        self.enabled = True
        self.phase = "prefill"
        self.first_decode: float | None = None
        self.capacity = capacity
        self._ring = None
        self._cursor = None
        self._k = None

    def _alloc(self, device, k: int) -> None:
        if self._ring is None or self._ring.device != device or self._k != k:
            self._k = k
            self._ring = torch.zeros(self.capacity, 3 + k, dtype=torch.int32, device=device)
            self._cursor = torch.zeros(1, dtype=torch.int64, device=device)

    def add(self, layer: int, topk_ids: torch.Tensor) -> None:
        if not self.enabled:
            return
        rows, k = topk_ids.shape
        if rows == 1 and self.first_decode is None:
            self.first_decode = time.perf_counter()
        self._alloc(topk_ids.device, k)
        ids = topk_ids.contiguous()
        _lib.call("d3_trace_append", _lib.ptr(ids), ids.element_size(), rows, k, int(layer),
                  _lib.ptr(self._ring), _lib.ptr(self._cursor), self.capacity,
                  _lib.stream_ptr())

    @property
    def dropped(self) -> int:
        if self._cursor is None:
            return 0
        return max(0, int(self._cursor.item()) - self.capacity)

    @property
    def records(self) -> list:
        if self._cursor is None:
            return []
        n = int(self._cursor.item())
        first = max(0, n - self.capacity)
        ring = self._ring.cpu()
        out, cur = [], None
        for r in range(first, n):
            row = ring[r % self.capacity].tolist()
            call, layer, phase, ids = row[0], row[1], row[2], row[3:]
            if cur is None or cur[0] != call:
                cur = (call, {"phase": "decode" if phase else "prefill", "layer": layer,
                              "ids": []})
                out.append(cur[1])
            cur[1]["ids"].append(ids)
        return out

    def save(self, path, meta: dict) -> None:
        import json
        from pathlib import Path
        Path(path).write_text(json.dumps({"meta": meta, "records": self.records}))


TRACE = RouterTrace()


# ---------------------------------------------------------------- census
# [layer, expert] call counts, prefill and decode together, and decode alone
# (one routed row); int64 device tensors (``.tolist()`` / ``.cpu()`` to read).
CENSUS = None
CENSUS_DECODE = None


def enable_census(layers: int = 40, experts: int = 256, device=None) -> None:
    global CENSUS, CENSUS_DECODE
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    CENSUS = torch.zeros(layers, experts, dtype=torch.int64, device=dev)
    CENSUS_DECODE = torch.zeros(layers, experts, dtype=torch.int64, device=dev)


def _count(layer: int, topk_ids: torch.Tensor) -> None:
    if CENSUS is None or layer < 0:
        return
    rows, k = topk_ids.shape
    ids = topk_ids.contiguous()
    _lib.call("d3_census_add", _lib.ptr(ids), ids.element_size(), rows, k, CENSUS.shape[1],
              _lib.ptr(CENSUS[layer]), _lib.ptr(CENSUS_DECODE[layer]), _lib.stream_ptr())


def observe(experts, topk_ids: torch.Tensor) -> None:
    """Census and trace of one MoE call (bin/offload.py:139-140)."""
    layer = getattr(experts, "_layer_index", -1)
    _count(layer, topk_ids)
    TRACE.add(layer, topk_ids)


def _buffers(experts, device):
    """Compact gather buffers for every expert of the layer shape, plus the plan
    tables; allocated once per (device, shape) and reused by every layer."""
    key = (device.index, tuple(experts.w13_weight.shape), tuple(experts.w2_weight.shape))
    b = _BUF.get(key)
    if b is None:
        E = experts.num_experts
        b = {
            "w13": torch.empty_like(experts.w13_weight, device=device),
            "w2": torch.empty_like(experts.w2_weight, device=device),
            "s13": torch.empty(experts.w13_scale_inv.shape, dtype=torch.float32, device=device),
            "s2": torch.empty(experts.w2_scale_inv.shape, dtype=torch.float32, device=device),
            "list": torch.empty(E, dtype=torch.int32, device=device),
            "n": torch.zeros(1, dtype=torch.int32, device=device),
            "remap": torch.empty(E, dtype=torch.int32, device=device),
        }
        b["dst"] = (ctypes.c_void_p * 4)(*(b[n].data_ptr() for n in ("w13", "w2", "s13", "s2")))
        _BUF[key] = b
    return b


def _layer_desc(experts):
    """The layer's device-cache descriptor, or a host-only one (no cache)."""
    d = getattr(experts, "_dc_desc", None)
    if d is not None and HYBRID_GATHER:
        return d
    from .devcache import _BUFFERS, _host_device_ptr
    hd = getattr(experts, "_d3_host_only_desc", None)
    if hd is None:
        hd = _lib.LayerCache()
        hd.num_experts = experts.num_experts
        hd.nbuf = 4
        for b, name in enumerate(_BUFFERS):
            t = getattr(experts, name)
            hd.host[b] = _host_device_ptr(t)
            hd.bytes[b] = t.numel() * t.element_size() // experts.num_experts
        experts._d3_host_only_desc = hd
    return hd


def gather_counters(experts) -> dict:
    c = getattr(experts, "_d3_gather_counters", None)
    if c is None:
        return {"gather_hits": 0, "gather_misses": 0}
    v = c.tolist()
    return {"gather_hits": v[0], "gather_misses": v[1]}


def offloaded_forward(self, x, topk_ids, topk_weights, fetch_ctas: int = 0):
    """MoE forward for experts held in pinned host memory (any number of rows).
    Layers installed with ``install_offload(..., chunk_prefetch=True)`` run
    through the model's shared ``ChunkPrefetch``."""
    pos = getattr(self, "_d3_chain_pos", None)
    if pos is not None and self.w13_weight.device.type == "cpu":
        pf = _CHAIN["pf"]
        if pf is None or pf.device != x.device:
            pf = _CHAIN["pf"] = ChunkPrefetch(_CHAIN["layers"], x.device)
        return pf.forward_in_order(pos, x, topk_ids, topk_weights)
    observe(self, topk_ids)
    return _union_forward(self, x, topk_ids, topk_weights, fetch_ctas)


def _union_forward(self, x, topk_ids, topk_weights, fetch_ctas: int = 0):
    """The layer's union of routed experts gathered after its router (cached
    ones borrowed read-only, the rest fetched), then the expert GEMM on the
    compact set (bin/offload.py:186-226)."""
    if self.w13_weight.device.type != "cpu":
        return moe.fp8_moe_forward(x, topk_ids, topk_weights, self.w13_weight,
                                   self.w13_scale_inv, self.w2_weight, self.w2_scale_inv)
    device = x.device
    T, k = topk_ids.shape
    E = self.num_experts
    b = _buffers(self, device)
    ids = topk_ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    local = torch.empty(T, k, dtype=torch.int32, device=device)
    st = _lib.stream_ptr()
    _lib.call("d3_prefill_plan", _lib.ptr(ids), ids.element_size(), ids.numel(), E,
              _lib.ptr(b["list"]), _lib.ptr(b["n"]), _lib.ptr(b["remap"]), _lib.ptr(local), st)
    cnt = getattr(self, "_d3_gather_counters", None)
    if cnt is None:
        cnt = torch.zeros(2, dtype=torch.int64, device=device)
        self._d3_gather_counters = cnt
    _lib.call("d3_gather_experts", ctypes.byref(_layer_desc(self)), _lib.ptr(b["list"]),
              _lib.ptr(b["n"]), b["dst"], _lib.ptr(cnt), int(fetch_ctas), st)
    if GATHER_DONE_HOOK is not None:
        GATHER_DONE_HOOK()
    return moe.fp8_moe_forward(x, local, topk_weights, b["w13"], b["s13"], b["w2"], b["s2"])


class ChunkPrefetch:
    """Prefill-chunk pipeline over a stack of offloaded layers: while layer
    l's expert GEMM runs, every expert of layer l+1 is gathered (cached ones
    borrowed read-only from that layer's device cache, the rest fetched from
    pinned host) into the other of two full-layer buffers, on a side stream.

    A 2048-token chunk routes top-8 to every one of the 256 experts of a layer
    (its union is the whole layer), so gathering the whole next layer fetches
    exactly the bytes the union gather of ``offloaded_forward`` would; the
    host link then never waits for a GEMM.  Below ``min_pairs_per_expert``
    routed pairs per expert (where the union is a fraction of the layer)
    ``forward`` falls back to ``offloaded_forward``.  Expert e sits at row e
    of the full-layer buffers, so the GEMM takes the routed ids as they are
    and gives the same bits as the union gather (whose compact numbering the
    GEMM's results do not depend on).

    Use: ``pf = ChunkPrefetch(layers)``; per chunk, for every layer in order,
    ``y = pf.forward(l, x, topk_ids, topk_weights)``.  Graph-capturable (the
    side stream forks from and joins the calling stream within each chunk).
    The reference gathers each layer's union after its router
    (bin/offload.py:186-226); it has no cross-layer prefetch."""

    def __init__(self, layers, device=None, fetch_ctas: int = 64,
                 min_pairs_per_expert: float = 4.0):
        self.layers = list(layers)
        ex0 = self.layers[0]
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.E = ex0.num_experts
        self.bufs = []
        for _ in range(2):
            b = {"w13": torch.empty(ex0.w13_weight.shape, dtype=ex0.w13_weight.dtype, device=dev),
                 "w2": torch.empty(ex0.w2_weight.shape, dtype=ex0.w2_weight.dtype, device=dev),
                 "s13": torch.empty(ex0.w13_scale_inv.shape, dtype=torch.float32, device=dev),
                 "s2": torch.empty(ex0.w2_scale_inv.shape, dtype=torch.float32, device=dev)}
            b["dst"] = (ctypes.c_void_p * 4)(*(b[n].data_ptr() for n in ("w13", "w2", "s13", "s2")))
            self.bufs.append(b)
        self.all = torch.arange(self.E, dtype=torch.int32, device=dev)
        self.n = torch.full((1,), self.E, dtype=torch.int32, device=dev)
        self.side = torch.cuda.Stream(device=dev)
        L = len(self.layers)
        self.ev_gathered = [torch.cuda.Event() for _ in range(L)]
        self.ev_used = [torch.cuda.Event() for _ in range(L)]
        self.fetch_ctas = int(fetch_ctas)
        self.min_pairs_per_expert = float(min_pairs_per_expert)
        self._piped = False
        self._next = -1
        for ex in self.layers:
            if getattr(ex, "_d3_gather_counters", None) is None:
                ex._d3_gather_counters = torch.zeros(2, dtype=torch.int64, device=dev)

    def _gather(self, l: int) -> None:
        ex = self.layers[l]
        b = self.bufs[l % 2]
        _lib.call("d3_gather_experts", ctypes.byref(_layer_desc(ex)), _lib.ptr(self.all),
                  _lib.ptr(self.n), b["dst"], _lib.ptr(ex._d3_gather_counters), self.fetch_ctas,
                  _lib.stream_ptr(self.side))
        self.ev_gathered[l].record(self.side)

    def forward(self, l: int, x, topk_ids, topk_weights):
        """Layer l's MoE output for the chunk (layers in order, l = 0 first)."""
        ex = self.layers[l]
        if l == 0:
            self._piped = (topk_ids.numel() >= self.min_pairs_per_expert * self.E
                           and ex.w13_weight.device.type == "cpu")
        if not self._piped or ex.w13_weight.device.type != "cpu":
            observe(ex, topk_ids)
            return _union_forward(ex, x, topk_ids, topk_weights)
        main = torch.cuda.current_stream(self.device)
        if l == 0:
            self.side.wait_stream(main)
            self._gather(0)
        if l + 1 < len(self.layers):
            if l >= 1:
                # the buffer layer l+1 lands in was read by layer l-1's GEMM
                self.side.wait_event(self.ev_used[l - 1])
            self._gather(l + 1)
        main.wait_event(self.ev_gathered[l])
        observe(ex, topk_ids)
        b = self.bufs[l % 2]
        y = moe.fp8_moe_forward(x, topk_ids, topk_weights, b["w13"], b["s13"], b["w2"], b["s2"])
        self.ev_used[l].record(main)
        return y

    def forward_in_order(self, l: int, x, topk_ids, topk_weights):
        """``forward`` for callers that see one layer at a time (the installed
        experts forward): layer 0 starts a chunk; a layer called out of order
        gathers its own union, and so does every later layer of that chunk.
        (Under stream capture an out-of-order call would leave the side
        stream's last gather unjoined, which the capture rejects.)"""
        if l == 0:
            self._next = 0
        if l != self._next:
            self._next = -1
            ex = self.layers[l]
            observe(ex, topk_ids)
            return _union_forward(ex, x, topk_ids, topk_weights)
        self._next = l + 1
        return self.forward(l, x, topk_ids, topk_weights)


def offloaded_stores(source) -> list:
    """The expert stores that live in host memory.  ``source`` is a model in
    the reference's layout (``model.backbone.model.layers[i].mlp.experts``:
    layers without an ``experts`` store, or whose store already sits on a
    GPU, are skipped) or any iterable of stores (``HostExperts``,
    ``OffloadedExperts.layers``)."""
    backbone = getattr(source, "backbone", None)
    if backbone is not None:
        found = (getattr(getattr(layer, "mlp", None), "experts", None)
                 for layer in backbone.model.layers)
    else:
        found = iter(source)
    return [ex for ex in found if ex is not None and ex.w13_weight.device.type == "cpu"]


def bytes_per_expert(experts) -> int:
    """Bytes one expert occupies over its four buffers (weights and scales),
    measured from the store itself -- the unit a cache slot holds."""
    from .devcache import _BUFFERS
    total = 0
    for name in _BUFFERS:
        t = getattr(experts, name)
        total += t.numel() * t.element_size() // experts.num_experts
    return total


def pin_experts(model, device=None) -> tuple[float, float]:
    """Page-lock every host expert buffer that is not page-locked yet
    (the reference's ``pin_experts``, bin/offload.py:664-699: same arguments,
    same (GiB newly pinned, seconds) result).  Buffers are replaced one at a
    time by a pinned copy, so the transient extra host memory is one buffer.
    ``model`` may also be an iterable of expert stores.  (The decode stack here
    uses ``hoststore.SharedHostStore`` instead: one page-locked copy per
    machine, registered in place.)"""
    from .devcache import _BUFFERS
    t0 = time.perf_counter()
    todo = [(ex, name) for ex in offloaded_stores(model) for name in _BUFFERS
            if not getattr(ex, name).is_pinned()]
    pinned_bytes = 0
    for ex, name in todo:
        locked = getattr(ex, name).pin_memory()
        setattr(ex, name, locked)
        pinned_bytes += locked.numel() * locked.element_size()
    return pinned_bytes / 2**30, time.perf_counter() - t0


def size_cache_to_free_vram(model, device, leave_free_gib: float = 2.0,
                            cap_per_layer: int = 256) -> int:
    """Give the device memory that is free right now, minus a reserve, to the
    expert caches of every offloaded layer, evenly (the reference's
    ``size_cache_to_free_vram``, bin/offload.py:611-661: same arguments and
    result).  The reserve is ``leave_free_gib`` for other programs plus
    ``ACTIVATION_HEADROOM_GIB`` for this process's own decode peak.  The
    allocator's idle blocks are released first so they count as free.  The
    slot size is measured from the stores (``bytes_per_expert``), and the
    capacity is clamped to ``cap_per_layer`` and to the layer's expert count.
    Allocates the caches (``devcache.init_dev_cache``) and returns the
    per-layer capacity; 0 (nothing allocated) when the budget does not hold
    one slot per layer."""
    from . import devcache
    stores = offloaded_stores(model)
    if not stores:
        return 0
    device = torch.device(device)
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()
    free_bytes = torch.cuda.mem_get_info(device)[0]
    reserve = int((leave_free_gib + ACTIVATION_HEADROOM_GIB) * 2**30)
    slot_row = sum(bytes_per_expert(ex) for ex in stores)   # one slot in every layer
    fits = max(0, free_bytes - reserve) // slot_row
    capacity = int(min(fits, cap_per_layer, min(ex.num_experts for ex in stores)))
    if capacity < 1:
        return 0
    for ex in stores:
        devcache.init_dev_cache(ex, device, capacity)
    return capacity


def install_offload(experts_cls, model=None, chunk_prefetch: bool = False) -> None:
    """Route ``experts_cls.forward`` through offloaded_forward, keeping the
    stock forward as ``_stock_forward`` (bin/offload.py:702-704).  With the
    model given, every layer's experts also get ``_layer_index`` (the census
    and trace key, bin/offload.py:128); with ``chunk_prefetch`` too, the
    offloaded layers share one ``ChunkPrefetch`` (multi-row calls gather the
    next layer's experts during this layer's GEMM; two full-layer buffers of
    device memory, ~1.6 GB at Drama-3's shapes, made on the first such call)."""
    experts_cls._stock_forward = experts_cls.forward
    experts_cls.forward = offloaded_forward
    if model is not None:
        chain = []
        for index, layer in enumerate(model.backbone.model.layers):
            experts = getattr(layer.mlp, "experts", None)
            if experts is not None:
                experts._layer_index = index
                if chunk_prefetch:
                    experts._d3_chain_pos = len(chain)
                    chain.append(experts)
        if chunk_prefetch:
            _CHAIN["layers"] = chain
            _CHAIN["pf"] = None
