"""Pin the CPU oracle to the reference's own kernels (no GPU).

The fixtures in tests/golden/resolve_golden.npz are outputs of the reference's
``_resolve_slots`` / ``_fetch_experts`` (bin/devcache.py:45-130) run under
TRITON_INTERPRET=1 by tests/golden/make_golden.py.
"""
import numpy as np
import pytest

import oracle
from conftest import GOLDEN

CASES = ["small_dups", "k_gt_c", "randperm_c16", "randperm_c32", "randperm_c64",
         "zipf_c51", "zipf_c68", "global_pool"]


@pytest.mark.parametrize("case", CASES)
def test_resolve_matches_reference(golden, case):
    g = lambda k: golden[f"{case}/{k}"]
    E, C = int(g("E")), int(g("C"))
    t = oracle.init_tables(E, C)
    for i, ids in enumerate(g("ids")):
        out, fs, fe, n = oracle.resolve(t, ids)
        assert n == int(g("nmiss")[i]), f"call {i}"
        np.testing.assert_array_equal(out, g("out")[i], err_msg=f"call {i}")
        np.testing.assert_array_equal(fs, g("fslot")[i][:n])
        np.testing.assert_array_equal(fe, g("fexp")[i][:n])
    np.testing.assert_array_equal(t.slot_of, g("final_slot_of"))
    np.testing.assert_array_equal(t.slot_expert, g("final_slot_expert"))
    np.testing.assert_array_equal(t.stamp, g("final_stamp"))
    np.testing.assert_array_equal(t.step, g("final_step"))


def test_fetch_matches_reference(golden):
    host = golden["fetch/host"]
    cache = np.full_like(golden["fetch/cache_after"], int(golden["fetch/fill"]))
    oracle.fetch(np.ascontiguousarray(host), cache, golden["fetch/fexp"], golden["fetch/fslot"],
                 int(golden["fetch/nmiss"][0]), host.shape[1])
    np.testing.assert_array_equal(cache, golden["fetch/cache_after"])
    # surplus jobs past nmiss left their slots untouched
    n = int(golden["fetch/nmiss"][0])
    for s in golden["fetch/fslot"][n:]:
        assert (cache[s] == int(golden["fetch/fill"])).all()


def test_replay_equals_stepwise(golden):
    """oracle.replay over a trace equals per-layer stepwise oracle.resolve."""
    from drama3_offloading_b200.trace import zipf_trace
    tr = zipf_trace(steps=64, layers=3)
    rep = oracle.replay(tr, 256, 20, want_slots=True)
    tabs = [oracle.init_tables(256, 20) for _ in range(3)]
    misses = 0
    for s in range(64):
        for l in range(3):
            out, _, _, n = oracle.resolve(tabs[l], tr[s, l])
            misses += n
            np.testing.assert_array_equal(out, rep["out_slots"][s, l])
    assert misses == rep["misses"]


def test_zipf_trace_golden_rows(golden):
    """The synthetic trace generator reproduces the rows the fixtures were made from."""
    from drama3_offloading_b200.trace import zipf_trace
    tr = zipf_trace(steps=200, layers=40)
    np.testing.assert_array_equal(tr[:, 0].astype(np.int32), golden["zipf_c51/ids"])
    np.testing.assert_array_equal(tr[:, 1].astype(np.int32), golden["zipf_c68/ids"])
    assert tr.dtype == np.int16 and tr.shape == (200, 40, 8)
    # top-k without replacement
    assert all(len(set(r.tolist())) == 8 for r in tr.reshape(-1, 8))
