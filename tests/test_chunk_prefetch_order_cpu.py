"""Host logic of offload.ChunkPrefetch.forward_in_order (no GPU): the order
rule that lets the installed experts forward, which sees one layer at a time,
drive the cross-layer prefill pipeline.  Layer 0 starts a chunk; layers in
order take the pipeline; a layer out of order, and every later layer of its
chunk, takes the union gather; the next layer 0 starts over."""
from drama3_offloading_b200 import offload


def _pipeline(monkeypatch):
    calls = []
    pf = object.__new__(offload.ChunkPrefetch)
    pf.layers = [f"layer{i}" for i in range(4)]
    pf._next = -1
    monkeypatch.setattr(pf, "forward", lambda l, x, i, w: calls.append(("pipe", l)) or "p",
                        raising=False)
    monkeypatch.setattr(offload, "_union_forward",
                        lambda ex, x, i, w: calls.append(("union", ex)) or "u")
    monkeypatch.setattr(offload, "observe", lambda ex, ids: None)
    return pf, calls


def test_in_order_chunks_take_the_pipeline(monkeypatch):
    pf, calls = _pipeline(monkeypatch)
    for _ in range(2):
        for l in range(4):
            assert pf.forward_in_order(l, None, None, None) == "p"
    assert calls == [("pipe", l) for l in range(4)] * 2


def test_out_of_order_falls_back_until_the_next_chunk(monkeypatch):
    pf, calls = _pipeline(monkeypatch)
    pf.forward_in_order(0, None, None, None)
    pf.forward_in_order(2, None, None, None)      # skipped layer 1
    pf.forward_in_order(3, None, None, None)      # the rest of the chunk too
    pf.forward_in_order(1, None, None, None)
    pf.forward_in_order(0, None, None, None)      # a new chunk starts over
    pf.forward_in_order(1, None, None, None)
    assert calls == [("pipe", 0), ("union", "layer2"), ("union", "layer3"),
                     ("union", "layer1"), ("pipe", 0), ("pipe", 1)]


def test_a_chunk_starting_mid_stack_takes_the_union(monkeypatch):
    pf, calls = _pipeline(monkeypatch)
    pf.forward_in_order(1, None, None, None)
    pf.forward_in_order(2, None, None, None)
    assert calls == [("union", "layer1"), ("union", "layer2")]
