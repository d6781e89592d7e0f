"""The allocator's LRU fast path (csrc/fetch.cu resolve_kernel), restated on
the CPU and checked against the oracle's sequential _resolve_slots on random
calls -- duplicates, out-of-range ids, small caches, Zipf routing -- and on
the decode trace.

The fast path resolves every hit at once and gives the misses, in id order,
the oldest slots that no hit of the call uses; the sequential rule gives a
miss the oldest slot not touched BEFORE it.  The two agree unless a slot hit
in the call is older than a chosen victim, which the fast path detects and
hands to the sequential loop.  This test checks that whenever the fast path
does not hand the call over, its slots, fetch jobs and final tables are the
oracle's, and counts how often it hands over."""
import random

import numpy as np

import oracle
from drama3_offloading_b200.trace import zipf_trace


def fast_path(slot_of, slot_expert, stamp, step, ids, n):
    """The kernel's fast path; None where it hands the call to the sequential loop."""
    k, C = len(ids), len(stamp)
    st = step + 1
    if k > 32 or k >= C:
        return None
    if not (-2**31 <= stamp.min() and stamp.max() < 2**31 and st < 2**31):
        return None
    valid = [0 <= e < n for e in ids]
    first = [next((j for j in range(i) if valid[j] and ids[j] == ids[i]), i) if valid[i] else i
             for i in range(k)]
    pre = [int(slot_of[ids[i]]) if valid[i] else -1 for i in range(k)]
    hit = [valid[i] and first[i] == i and pre[i] >= 0 and slot_expert[pre[i]] == ids[i]
           for i in range(k)]
    mark = np.zeros(C, np.int32)
    for i in range(k):
        if hit[i]:
            mark[pre[i]] = 1
    misses = [i for i in range(k) if valid[i] and first[i] == i and not hit[i]]
    if len(misses) > C - int(mark.sum()):
        return None
    vict = []
    for _ in misses:
        _, c = min((int(stamp[c]), c) for c in range(C) if mark[c] == 0)
        vict.append(c)
        mark[c] = 2
    if misses and any(hit):
        if min((int(stamp[pre[i]]), pre[i]) for i in range(k) if hit[i]) < \
                (int(stamp[vict[-1]]), vict[-1]):
            return None
    so, se, sp = slot_of.copy(), slot_expert.copy(), stamp.copy()
    out = [-1] * k
    for r, i in enumerate(misses):
        v = vict[r]
        if se[v] >= 0:
            so[se[v]] = -1
        so[ids[i]], se[v] = v, ids[i]
    for i in range(k):
        if valid[i] and first[i] == i:
            out[i] = pre[i] if hit[i] else vict[misses.index(i)]
            sp[out[i]] = st
    for i in range(k):
        if valid[i] and first[i] != i:
            out[i] = out[first[i]]
    return out, vict, [ids[i] for i in misses], so, se, sp


def _check(t, ids, n):
    so, se, sp, stp = t.slot_of.copy(), t.slot_expert.copy(), t.stamp.copy(), int(t.step[0])
    fast = fast_path(so, se, sp, stp, ids, n)
    # oracle on the in-range ids (the kernel skips the others: slot -1, no fetch)
    keep = [i for i, e in enumerate(ids) if 0 <= e < n]
    out, fs, fe, nm = oracle.resolve(t, np.array([ids[i] for i in keep], np.int32))
    if fast is None:
        return False
    want = [-1] * len(ids)
    for j, i in enumerate(keep):
        want[i] = int(out[j])
    assert fast[0] == want, (ids, fast[0], want)
    assert fast[1] == list(fs) and fast[2] == list(fe)
    assert (fast[3] == t.slot_of).all() and (fast[4] == t.slot_expert).all()
    assert (fast[5] == t.stamp).all()
    return True


def test_fast_path_matches_the_sequential_oracle_on_random_calls():
    rng = random.Random(1)
    taken = total = 0
    for _ in range(400):
        n = rng.choice([16, 64, 256])
        C = min(n, rng.choice([9, 12, 16, 33, 68, 100]))
        k = min(rng.choice([1, 2, 3, 8, 8, 16, 31]), C - 1)
        t = oracle.init_tables(n, C)
        zipf = rng.random() < 0.7
        for _ in range(rng.randint(1, 40)):
            if zipf:
                ids = [min(n - 1, int(rng.paretovariate(1.1))) for _ in range(k)]
            else:
                ids = [rng.randrange(n) for _ in range(k)]
            if rng.random() < 0.05:
                ids[rng.randrange(k)] = n + 3          # out of range: skipped
            taken += _check(t, ids, n)
            total += 1
    assert taken > 0.85 * total, (taken, total)


def test_fast_path_on_the_decode_trace():
    tr = zipf_trace(steps=300, layers=4, seed=0)
    taken = total = 0
    for l in range(4):
        t = oracle.init_tables(256, 68)
        for s in range(tr.shape[0]):
            taken += _check(t, [int(x) for x in tr[s, l]], 256)
            total += 1
    assert taken > 0.9 * total, (taken, total)
