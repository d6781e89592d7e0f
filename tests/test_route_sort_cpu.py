"""The route launch's parallel stable sort (csrc/moe.cu route_kernel),
restated on the CPU: NW warps over consecutive chunks of the pairs, per-chunk
expert histograms, a column scan into chunk-local bases, then placement at
off[e] + base[w][e] + rank among equal ids in the 32-pair batch.  It must
give exactly the order of a sequential stable counting sort (pairs of one
expert in pair order), which is what the GEMM tiles and the combine's
fixed summation order rely on."""
import random

import numpy as np
import pytest


def chunk(P: int, nw: int) -> int:
    batches = (P + 31) // 32
    return (batches + nw - 1) // nw * 32


def route_sort(ids: np.ndarray, n: int, nw: int):
    P = len(ids)
    C = chunk(P, nw)
    valid = lambda e: 0 <= e < n
    hist = np.zeros((nw, n), dtype=np.int64)
    for w in range(nw):                                   # pass 1
        for i in range(w * C, min(P, (w + 1) * C)):
            if valid(ids[i]):
                hist[w, ids[i]] += 1
    cnt = hist.sum(0)
    base = np.zeros_like(hist)                            # column scan
    base[1:] = np.cumsum(hist, 0)[:-1]
    off = np.concatenate([[0], np.cumsum(cnt)[:-1]])      # block scan
    sorted_ = np.full(P, -1, dtype=np.int64)
    inv = np.full(P, -1, dtype=np.int64)
    for w in range(nw):                                   # pass 2
        cur = base[w].copy()
        for b0 in range(w * C, min(P, (w + 1) * C), 32):
            batch = list(range(b0, min(b0 + 32, P, (w + 1) * C)))
            for lane, i in enumerate(batch):
                e = ids[i]
                if not valid(e):
                    continue
                rank = sum(1 for i2 in batch[:lane] if ids[i2] == e)
                pos = off[e] + cur[e] + rank
                sorted_[pos] = i
                inv[i] = pos
            for i in batch:                               # the leaders' cursor updates
                if valid(ids[i]):
                    cur[ids[i]] += 1
    return sorted_, inv, cnt, off


def reference_sort(ids: np.ndarray, n: int):
    order = [i for e in range(n) for i in range(len(ids)) if ids[i] == e]
    P = len(ids)
    sorted_ = np.full(P, -1, dtype=np.int64)
    inv = np.full(P, -1, dtype=np.int64)
    for pos, i in enumerate(order):
        sorted_[pos] = i
        inv[i] = pos
    return sorted_, inv


@pytest.mark.parametrize("P,n,nw", [(8, 256, 1), (512, 32, 16), (40, 256, 2), (1000, 64, 32),
                                    (4096, 256, 32), (33, 8, 3), (64, 8192, 1)])
def test_matches_sequential_stable_sort(P, n, nw):
    rng = np.random.default_rng(P * 7 + n + nw)
    ids = rng.integers(-2, n + 2, size=P)   # with out-of-range (skipped) ids
    got_sorted, got_inv, cnt, off = route_sort(ids, n, min(nw, (P + 31) // 32))
    want_sorted, want_inv = reference_sort(ids, n)
    assert np.array_equal(got_sorted, want_sorted)
    assert np.array_equal(got_inv, want_inv)
    assert int(cnt.sum()) == int(((ids >= 0) & (ids < n)).sum())


def test_random_shapes():
    r = random.Random(3)
    for _ in range(60):
        P, n = r.randint(1, 700), r.randint(1, 300)
        nw = r.randint(1, 32)
        ids = np.array([r.randint(-1, n) for _ in range(P)])
        got_sorted, got_inv, _, _ = route_sort(ids, n, min(nw, (P + 31) // 32))
        want_sorted, want_inv = reference_sort(ids, n)
        assert np.array_equal(got_sorted, want_sorted) and np.array_equal(got_inv, want_inv)
