"""Device-side routing census and router trace (bin/offload.py:40-79 and
:257-287 restated on the device), through the C ABI and the offload module's
reference-named API: counts equal numpy's bincount of the same ids, decode
counts take one-row calls only, out-of-range ids are not counted, graph
replays keep counting, and the trace ring reproduces the per-call records
(phase, layer, ids) and keeps the newest rows when it wraps."""
import numpy as np
import pytest
import torch

from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import offload  # noqa: E402

DEV = torch.device("cuda:0")


class _Layer:
    def __init__(self, index):
        self._layer_index = index


def test_census_matches_bincount():
    offload.enable_census(layers=3, experts=64, device=DEV)
    g = torch.Generator().manual_seed(0)
    want = np.zeros((3, 64), np.int64)
    want_dec = np.zeros((3, 64), np.int64)
    for step in range(20):
        rows = 1 if step % 3 else 17
        layer = step % 3
        ids = torch.randint(-2, 70, (rows, 8), generator=g)  # some out of range
        dtype = torch.int64 if step % 2 else torch.int32
        offload._count(layer, ids.to(dtype).to(DEV))
        valid = ids[(ids >= 0) & (ids < 64)].numpy()
        c = np.bincount(valid, minlength=64)
        want[layer] += c
        if rows == 1:
            want_dec[layer] += c
    torch.cuda.synchronize()
    np.testing.assert_array_equal(offload.CENSUS.cpu().numpy(), want)
    np.testing.assert_array_equal(offload.CENSUS_DECODE.cpu().numpy(), want_dec)
    offload.CENSUS = offload.CENSUS_DECODE = None


def test_census_counts_every_graph_replay():
    offload.enable_census(layers=1, experts=16, device=DEV)
    ids = torch.tensor([[1, 2, 3, 3, 15, 0, 7, 8]], dtype=torch.int32, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        offload._count(0, ids)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        offload._count(0, ids)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    want = np.bincount(ids.cpu().numpy().ravel(), minlength=16) * 4   # warm-up + 3 replays
    np.testing.assert_array_equal(offload.CENSUS[0].cpu().numpy(), want)
    np.testing.assert_array_equal(offload.CENSUS_DECODE[0].cpu().numpy(), want)
    offload.CENSUS = offload.CENSUS_DECODE = None


def test_trace_records_and_wrap():
    tr = offload.RouterTrace(capacity=64)
    g = torch.Generator().manual_seed(1)
    calls = []
    for c in range(12):
        rows = 1 if c % 4 else 5
        ids = torch.randint(0, 256, (rows, 8), generator=g, dtype=torch.int32)
        tr.add(c % 40, ids.to(DEV))
        calls.append({"phase": "decode" if rows == 1 else "prefill", "layer": c % 40,
                      "ids": ids.tolist()})
    recs = tr.records
    assert tr.dropped == 0
    assert recs == calls
    # wrap: a ring of 6 rows keeps the newest 6
    small = offload.RouterTrace(capacity=6)
    rows_in = []
    for c in range(5):
        ids = torch.full((2, 8), c, dtype=torch.int64)
        small.add(7, ids.to(DEV))
        rows_in += ids.tolist()
    assert small.dropped == 4
    kept = [r for rec in small.records for r in rec["ids"]]
    assert kept == rows_in[-6:]
    assert all(rec["layer"] == 7 and rec["phase"] == "prefill" for rec in small.records)


def test_offloaded_forward_hook_observes():
    """observe() keys the census and the trace by the experts' _layer_index."""
    offload.enable_census(layers=4, experts=32, device=DEV)
    old = offload.TRACE
    offload.TRACE = offload.RouterTrace(capacity=16)
    try:
        ids = torch.tensor([[3, 4, 5, 6, 7, 8, 9, 10]], dtype=torch.int32, device=DEV)
        offload.observe(_Layer(2), ids)
        offload.observe(_Layer(-1), ids)      # no index: not counted, traced as layer -1
        torch.cuda.synchronize()
        assert int(offload.CENSUS[2].sum()) == 8 and int(offload.CENSUS.sum()) == 8
        assert [r["layer"] for r in offload.TRACE.records] == [2, -1]
        assert offload.TRACE.first_decode is not None
    finally:
        offload.TRACE = old
        offload.CENSUS = offload.CENSUS_DECODE = None
