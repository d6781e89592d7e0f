"""The allocator oracle on the reference's own captured decode routing
(211 frames x 40 layers x top-8, tests/golden/route_trace_512.npz, made by
make_trace_golden.py from notes/route-trace-512.json):

* LRU (the reference's _resolve_slots semantics, which the oracle matches bit
  for bit on the golden allocator cases) reproduces the reference's published
  per-layer LRU hit rates -- 70.6 / 77.9 / 80.7 / 86.4 % at 85 / 113 / 127 /
  170 experts per layer (notes/02-first-results.md:65-72) -- to the published
  decimal, and the reference simulator's (bin/simulate_cache.py:64-97) hit
  counts within 0.1 points (the simulator's OrderedDict breaks equal-age ties
  by access order, _resolve_slots by lowest slot index).
* LFU: the device policy may not evict a slot already promised to an id of
  the same call (the expert GEMM reads it next), which the simulator's LFU
  does; on this trace that never loses hits against it.
"""
from pathlib import Path

import numpy as np

import oracle

FIX = Path(__file__).resolve().parent / "golden" / "route_trace_512.npz"
PUBLISHED_LRU = {85: 70.6, 113: 77.9, 127: 80.7, 170: 86.4}


def _rate(r) -> float:
    return r["hits"] / (r["hits"] + r["misses"])


def test_lru_reproduces_the_published_hit_rates():
    f = np.load(FIX)
    trace = f["trace"]
    assert trace.shape == (211, 40, 8)
    for cap, ref_hits, total in zip(f["caps"], f["ref_lru_hits"], f["total"]):
        r = oracle.replay(trace, 256, int(cap), "lru")
        assert r["hits"] + r["misses"] == total
        assert abs(_rate(r) - ref_hits / total) < 1e-3, cap
        if int(cap) in PUBLISHED_LRU:
            assert round(100 * _rate(r), 1) == PUBLISHED_LRU[int(cap)], cap


def test_lfu_never_below_the_reference_simulator():
    f = np.load(FIX)
    for cap, ref_hits, total in zip(f["caps"], f["ref_lfu_hits"], f["total"]):
        r = oracle.replay(f["trace"], 256, int(cap), "lfu")
        assert r["hits"] >= ref_hits, cap
