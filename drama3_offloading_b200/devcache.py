"""Device-resident expert cache -- drop-in for the reference's ``bin/devcache.py``.

Same public surface and attribute names as the reference module, so code that
imports ``devcache`` (``bin/narrate.py:635-650``, ``bin/server.py:312-324``,
``bin/offload.py:201-207``, ``bin/prefill_probe.py:77``) works unchanged:

* ``init_dev_cache(experts, device, capacity)``      (bin/devcache.py:138-167)
* ``dev_resolve_and_fetch(experts, topk_ids)``        (bin/devcache.py:230-255)
* ``dev_cached_forward(self, x, topk_ids, topk_weights)`` (bin/devcache.py:258-277)
* ``install_dev_cache(model, device, capacity)``      (bin/devcache.py:280-301)
* ``EXPERT_BYTES``, ``FETCH_BACKEND``, ``CPP_BLOCKS_PER_JOB`` and the per-layer
  attributes ``_dc_cap, _dc_slot_of, _dc_slot_expert, _dc_stamp, _dc_step,
  _dc_w13, _dc_w2, _dc_s13, _dc_s2, _dc_out, _dc_fslot, _dc_fexp, _dc_nmiss``.

All work runs in libd3b200.so (sm_100a): there is no Triton path and no CPU
fallback.  ``FETCH_BACKEND``:

* ``"b200"`` (default) -- one allocator launch plus ONE fetch launch that moves
  all four buffers of every miss (``d3_resolve_fetch``).
* ``"cpp"``  -- the reference's launch sequence (allocator, then one fetch per
  buffer, ``CPP_BLOCKS_PER_JOB`` CTAs per job) on this library's kernels
  (``d3_resolve_slots`` + ``d3_fetch_experts``), kept for A/B comparison.

Decode steps (one routed row) of ``dev_cached_forward`` go through
``dev_resolve_fetch_moe`` when ``OVERLAP`` is on (default, ``"b200"`` only):
the allocator launch, then ONE launch that fetches the misses on a few CTAs
while the others run the gate/up products of the resident experts (and of the
shared expert) and then of each fetched expert as soon as its bytes have
landed, then the down projection (``d3_resolve_fetch_moe``).  Same slots,
same bits as resolve + fetch followed by ``moe.fp8_moe_forward``.

``"triton"`` is rejected with ValueError.  Every call is sync-free and keeps a
static launch shape, so it can be captured into a CUDA graph and replayed with
new ids (the slot table, step counter and job count live on the device).

Additions over the reference: ``POLICY`` ("lru" = the reference's allocator,
bit-exact; "lfu" = frequency eviction) and ``_dc_counters`` -- cumulative
device-side {calls, hits, misses, bytes fetched}, read with ``stats()``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

EXPERT_BYTES = 3_146_496
FETCH_BACKEND = "b200"
CPP_BLOCKS_PER_JOB = 64
FETCH_CTAS = 0          # fused fetch grid; 0 = one CTA per SM
OVERLAP = True          # decode: fetch + gate/up in one launch (d3_resolve_fetch_moe)
OVERLAP_FETCH_CTAS = 64  # CTAs that fetch inside that launch; the rest run the gate/up units
POLICY = "lru"
K_MAX = 64              # largest k one resolve call accepts

_BUFFERS = ("w13_weight", "w2_weight", "w13_scale_inv", "w2_scale_inv")


def _host_device_ptr(t: torch.Tensor) -> int:
    """Device-visible base of a pinned CPU tensor (D3_ERR_NOT_PINNED otherwise)."""
    if t.device.type != "cpu" or not t.is_contiguous():
        raise RuntimeError("expected a contiguous page-locked CPU tensor")
    out = ctypes.c_void_p(0)
    _lib.call("d3_device_ptr_of", ctypes.c_void_p(t.data_ptr()),
              ctypes.c_size_t(t.numel() * t.element_size()), ctypes.byref(out))
    return int(out.value or 0)


def init_dev_cache(experts, device: torch.device, capacity: int, policy: str | None = None) -> None:
    """Allocate one layer's device cache and slot tables (bin/devcache.py:138-167).

    Slot tables start as the reference's: ``slot_of = -1``, ``slot_expert = -1``,
    ``stamp = -(C..1)`` (first C misses fill slots 0,1,2,...), ``step = 0``.
    Weight slots are zero, scale slots one (a stale read degrades to silence).
    """
    device = torch.device(device)
    policy = (policy or POLICY).lower()
    if policy not in ("lru", "lfu"):
        raise ValueError(f"policy must be 'lru' or 'lfu', got {policy!r}")
    n_experts = experts.num_experts
    if not (1 <= capacity <= 8192):
        raise ValueError(f"capacity must be in [1, 8192], got {capacity}")
    experts._dc_cap = capacity
    experts._dc_policy = policy
    experts._dc_slot_of = torch.full((n_experts,), -1, dtype=torch.int32, device=device)
    experts._dc_slot_expert = torch.full((capacity,), -1, dtype=torch.int32, device=device)
    experts._dc_stamp = -torch.arange(capacity, 0, -1, dtype=torch.int64, device=device)
    experts._dc_step = torch.zeros(1, dtype=torch.int64, device=device)
    experts._dc_freq = torch.zeros(capacity, dtype=torch.int64, device=device)
    experts._dc_ins = -torch.arange(capacity, 0, -1, dtype=torch.int64, device=device)

    def buf(src, fill):
        return torch.full((capacity, *src.shape[1:]), fill, dtype=src.dtype, device=device)

    experts._dc_w13 = buf(experts.w13_weight, 0)
    experts._dc_w2 = buf(experts.w2_weight, 0)
    experts._dc_s13 = torch.ones((capacity, *experts.w13_scale_inv.shape[1:]),
                                 dtype=torch.float32, device=device)
    experts._dc_s2 = torch.ones((capacity, *experts.w2_scale_inv.shape[1:]),
                                dtype=torch.float32, device=device)
    # per-call result and job tables live here for the layer's lifetime: a
    # resolve call writes into them and never allocates, so it can be captured
    experts._dc_out = torch.zeros(K_MAX, dtype=torch.int32, device=device)
    experts._dc_fslot = torch.zeros(K_MAX, dtype=torch.int32, device=device)
    experts._dc_fexp = torch.zeros(K_MAX, dtype=torch.int32, device=device)
    experts._dc_nmiss = torch.zeros(1, dtype=torch.int32, device=device)
    experts._dc_counters = torch.zeros(4, dtype=torch.int64, device=device)

    desc = _lib.LayerCache()
    desc.num_experts = n_experts
    desc.capacity = capacity
    desc.policy = _lib.D3_POLICY_LFU if policy == "lfu" else _lib.D3_POLICY_LRU
    desc.nbuf = 4
    for name in ("slot_of", "slot_expert", "stamp", "step", "freq", "ins"):
        setattr(desc, name, getattr(experts, f"_dc_{name}").data_ptr())
    desc.out_slot = experts._dc_out.data_ptr()
    desc.fetch_slot = experts._dc_fslot.data_ptr()
    desc.fetch_expert = experts._dc_fexp.data_ptr()
    desc.nmiss = experts._dc_nmiss.data_ptr()
    desc.counters = experts._dc_counters.data_ptr()
    host_ptrs = []
    for b, (name, cache) in enumerate(zip(_BUFFERS, (experts._dc_w13, experts._dc_w2,
                                                     experts._dc_s13, experts._dc_s2))):
        host = getattr(experts, name)
        per = host.numel() * host.element_size() // n_experts
        if per % 16:
            raise ValueError(f"{name}: {per} bytes per expert is not a multiple of 16")
        hp = _host_device_ptr(host)
        host_ptrs.append(hp)
        desc.host[b] = hp
        desc.cache[b] = cache.data_ptr()
        desc.bytes[b] = per
    experts._dc_host_ptrs = host_ptrs
    experts._dc_desc = desc


def reset_dev_cache(experts) -> None:
    """Return one layer's tables to the init_dev_cache state in place (same
    device addresses, so captured graphs stay valid); slot bytes are left as
    they are -- no slot is referenced any more."""
    C = experts._dc_cap
    experts._dc_slot_of.fill_(-1)
    experts._dc_slot_expert.fill_(-1)
    torch.arange(C, 0, -1, dtype=torch.int64, device=experts._dc_stamp.device,
                 out=experts._dc_stamp).neg_()
    experts._dc_step.zero_()
    experts._dc_freq.zero_()
    experts._dc_ins.copy_(experts._dc_stamp)
    experts._dc_nmiss.zero_()
    experts._dc_counters.zero_()


def _copy_pairs(experts):
    """(host device-pointer, cache tensor, bytes per expert) for the 4 buffers
    (bin/devcache.py:170-181)."""
    d = experts._dc_desc
    return [(d.host[b], c, d.bytes[b]) for b, c in enumerate(
        (experts._dc_w13, experts._dc_w2, experts._dc_s13, experts._dc_s2))]


def _ids_arg(topk_ids: torch.Tensor) -> torch.Tensor:
    ids = topk_ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    return ids.contiguous()


def dev_resolve_and_fetch(experts, topk_ids: torch.Tensor, stream=None) -> torch.Tensor:
    """Resolve ids to slots, fetching misses. Returns int32 slots [k], no sync."""
    ids = _ids_arg(topk_ids)
    k = ids.numel()
    if not (1 <= k <= K_MAX):
        raise ValueError(f"resolve takes 1..{K_MAX} ids per call, got {k}")
    st = _lib.stream_ptr(stream)
    if FETCH_BACKEND == "b200":
        _lib.call("d3_resolve_fetch", ctypes.byref(experts._dc_desc), _lib.ptr(ids),
                  ids.element_size(), k, int(FETCH_CTAS), st)
    elif FETCH_BACKEND == "cpp":
        _lib.call("d3_resolve_slots", _lib.ptr(ids), ids.element_size(), k,
                  _lib.ptr(experts._dc_slot_of), experts.num_experts,
                  _lib.ptr(experts._dc_slot_expert), _lib.ptr(experts._dc_stamp),
                  experts._dc_cap, _lib.ptr(experts._dc_out), _lib.ptr(experts._dc_fslot),
                  _lib.ptr(experts._dc_fexp), _lib.ptr(experts._dc_nmiss),
                  _lib.ptr(experts._dc_step), st)
        for host, cache, per in _copy_pairs(experts):
            bpj = CPP_BLOCKS_PER_JOB if per >= 65536 else 1
            _lib.call("d3_fetch_experts", ctypes.c_void_p(host), _lib.ptr(cache),
                      _lib.ptr(experts._dc_fexp), _lib.ptr(experts._dc_fslot),
                      _lib.ptr(experts._dc_nmiss), per, k, bpj, 256, st)
    else:
        raise ValueError(f"FETCH_BACKEND must be 'b200' or 'cpp' (no Triton path), "
                         f"got {FETCH_BACKEND!r}")
    return experts._dc_out[:k]


def dev_resolve_fetch_moe(experts, topk_ids: torch.Tensor, x: torch.Tensor,
                          topk_weights: torch.Tensor, out: torch.Tensor | None = None,
                          accumulate: bool = False, shared: tuple | None = None,
                          stream=None, stages: int = 7, l2_warm=None,
                          l2_warm_bytes=None) -> torch.Tensor:
    """One decode row through the cache: resolve ``topk_ids`` [1, k], fetch the
    misses while the gate/up products of the resident experts run, then the
    down projection into ``out`` (bf16 [1, H]; added to it with
    ``accumulate``).  ``shared=(w13_s, w2_s, gate_s)`` adds the shared expert
    inside the same launches.  Sync-free and graph-capturable.  ``stages``
    masks the launches issued (1 allocator, 2 fetch + gate/up, 4 down
    projection; 7 = all), to time them apart.  ``l2_warm``: a contiguous
    device tensor, or a list of up to 4, of static weights the next launches
    read (e.g. the next layer's router gate and dense weights); the first
    ``l2_warm_bytes`` (an int, or one per tensor; None = all) of each are
    hinted into L2 while the fetch holds the host link."""
    from . import moe
    ids = _ids_arg(topk_ids)
    k = ids.numel()
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[0] != 1 or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 [1, H] row")
    H = x.shape[1]
    I = experts._dc_w2.shape[2]
    w = topk_weights.reshape(k)
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.to(torch.float32)
    w = w.contiguous()
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs an out tensor")
        out = torch.empty(1, H, dtype=torch.bfloat16, device=x.device)
    sw13 = sw2 = sg = None
    if shared is not None:
        sw13, sw2, sg = shared
    need = int(_lib.load().d3_resolve_fetch_moe_workspace_size(k, H, I))
    if need == 0:
        raise ValueError(f"unsupported shape k={k} H={H} I={I}")
    ws = moe._workspace(x.device, need, "overlap")
    args = (ctypes.byref(experts._dc_desc), _lib.ptr(ids),
            ids.element_size(), k, _lib.ptr(x), _lib.ptr(w),
            1 if w.dtype == torch.float32 else 0, H, I,
            _lib.ptr(sw13) if sw13 is not None else None,
            _lib.ptr(sw2) if sw2 is not None else None,
            _lib.ptr(sg) if sg is not None else None, _lib.ptr(out), 1 if accumulate else 0,
            _lib.ptr(moe.error_word(x.device)), _lib.ptr(ws), ws.numel(),
            int(OVERLAP_FETCH_CTAS), int(stages))
    if l2_warm is None:
        _lib.call("d3_resolve_fetch_moe", *args, _lib.stream_ptr(stream))
    else:
        ts = list(l2_warm) if isinstance(l2_warm, (list, tuple)) else [l2_warm]
        caps = (list(l2_warm_bytes) if isinstance(l2_warm_bytes, (list, tuple))
                else [l2_warm_bytes] * len(ts))
        if not 1 <= len(ts) <= 4 or len(caps) != len(ts):
            raise ValueError("l2_warm: 1 to 4 tensors, l2_warm_bytes one per tensor")
        ptrs = (ctypes.c_void_p * len(ts))()
        nbs = (ctypes.c_size_t * len(ts))()
        for i, (t, cap) in enumerate(zip(ts, caps)):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError("l2_warm tensors must be contiguous device tensors")
            nb = t.numel() * t.element_size()
            ptrs[i] = t.data_ptr()
            nbs[i] = nb if cap is None else max(0, min(nb, int(cap)))
        _lib.call("d3_resolve_fetch_moe_l2warm", *args, ptrs, nbs, len(ts),
                  _lib.stream_ptr(stream))
    return out


def _overlap_ok(experts, topk_ids, x) -> bool:
    H = x.shape[-1]
    I = experts._dc_w2.shape[2]
    return (OVERLAP and FETCH_BACKEND == "b200" and x.dim() == 2 and x.shape[0] == 1
            and H % 512 == 0 and I % 512 == 0 and experts._dc_cap >= topk_ids.numel())


def dev_cached_forward(self, x, topk_ids, topk_weights):
    """``MoEExperts.forward`` through the device cache (bin/devcache.py:258-277).

    Decode (one routed row) resolves + fetches on device and runs the FP8
    grouped expert GEMM over the cache slots; prefill (several rows) goes to
    ``offload.offloaded_forward``, the gather path with a read-only borrow from
    this cache."""
    from . import moe
    if topk_ids.shape[0] != 1 or not getattr(self, "_dc_cap", 0):
        from . import offload
        return offload.offloaded_forward(self, x, topk_ids, topk_weights)
    if _overlap_ok(self, topk_ids, x):
        return dev_resolve_fetch_moe(self, topk_ids, x.contiguous(), topk_weights)
    slots = dev_resolve_and_fetch(self, topk_ids)
    return moe.fp8_moe_forward(x, slots.reshape(topk_ids.shape), topk_weights, self._dc_w13,
                               self._dc_s13, self._dc_w2, self._dc_s2)


def install_dev_cache(model, device, capacity: int) -> int:
    """Allocate the device cache on every offloaded layer and swap in the
    forward (bin/devcache.py:280-301).  Raises RuntimeError unless the host
    expert tensors are page-locked.  Returns the number of layers."""
    n = 0
    classes = set()
    for layer in model.backbone.model.layers:
        experts = getattr(layer.mlp, "experts", None)
        if experts is None or experts.w13_weight.device.type != "cpu":
            continue
        if not experts.w13_weight.is_pinned():
            raise RuntimeError(
                "device cache needs pinned expert tensors; run pin_experts first")
        init_dev_cache(experts, device, capacity)
        classes.add(type(experts))
        n += 1
    for cls in classes:
        cls.forward = dev_cached_forward
    return n


def stats(experts) -> dict:
    """Cumulative device counters of one layer (synchronises; not for the hot loop)."""
    c = experts._dc_counters.tolist()
    return {"calls": c[0], "hits": c[1], "misses": c[2], "bytes_fetched": c[3]}
