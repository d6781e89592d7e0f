"""Prefill gather on the GPU, through the C ABI: the device-side union/remap
(replacing torch.unique(ids.cpu()), bin/offload.py:157-158), the one-launch
hybrid gather (cached experts borrowed read-only from the device cache, the
rest fetched from pinned host, bin/offload.py:186-226) with self-identifying
bytes, and offloaded_forward against the all-resident path and the oracle."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import _lib, devcache, moe, offload, synth  # noqa: E402

DEV = torch.device("cuda:0")


def test_prefill_plan_matches_unique():
    g = torch.Generator().manual_seed(5)
    E = 256
    ids = torch.randint(0, E, (300, 8), generator=g, dtype=torch.int32)
    ids[0, 0] = -1
    ids[1, 1] = E + 3
    d = ids.to(DEV)
    lst = torch.empty(E, dtype=torch.int32, device=DEV)
    n = torch.zeros(1, dtype=torch.int32, device=DEV)
    remap = torch.empty(E, dtype=torch.int32, device=DEV)
    local = torch.empty_like(d)
    _lib.call("d3_prefill_plan", _lib.ptr(d), 4, d.numel(), E, _lib.ptr(lst), _lib.ptr(n),
              _lib.ptr(remap), _lib.ptr(local), _lib.stream_ptr())
    torch.cuda.synchronize()
    flat = ids.reshape(-1).numpy()
    valid = flat[(flat >= 0) & (flat < E)]
    uniq = np.unique(valid)
    assert int(n.item()) == len(uniq)
    np.testing.assert_array_equal(lst.cpu().numpy()[:len(uniq)], uniq)
    want_remap = np.full(E, -1)
    want_remap[uniq] = np.arange(len(uniq))
    np.testing.assert_array_equal(remap.cpu().numpy(), want_remap)
    want_local = np.where((flat >= 0) & (flat < E), want_remap[np.clip(flat, 0, E - 1)], -1)
    np.testing.assert_array_equal(local.cpu().numpy().reshape(-1), want_local)


@pytest.fixture(scope="module")
def pattern_host():
    return synth.pattern_experts(64)


def test_gather_borrows_read_only_and_fetches_misses(pattern_host):
    ex = synth.HostExperts(64, pattern_host.w13_weight, pattern_host.w2_weight,
                           pattern_host.w13_scale_inv, pattern_host.w2_scale_inv)
    devcache.init_dev_cache(ex, DEV, 16)
    # make experts 0..7 resident
    devcache.dev_resolve_and_fetch(ex, torch.arange(8, dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    stamp0 = ex._dc_stamp.clone()
    step0 = ex._dc_step.clone()
    slot_of0 = ex._dc_slot_of.clone()
    ids = torch.tensor([[3, 40, 5], [40, 12, 63], [0, 5, 12]], dtype=torch.int32, device=DEV)
    x = torch.randn(3, 2048, device=DEV).to(torch.bfloat16)
    b = offload._buffers(ex, DEV)
    offload.offloaded_forward  # noqa: B018 (the function under test below uses these)
    lst = b["list"]
    local = torch.empty_like(ids)
    st = _lib.stream_ptr()
    _lib.call("d3_prefill_plan", _lib.ptr(ids), 4, ids.numel(), 64, _lib.ptr(lst),
              _lib.ptr(b["n"]), _lib.ptr(b["remap"]), _lib.ptr(local), st)
    cnt = torch.zeros(2, dtype=torch.int64, device=DEV)
    _lib.call("d3_gather_experts", ctypes.byref(ex._dc_desc), _lib.ptr(lst), _lib.ptr(b["n"]),
              b["dst"], _lib.ptr(cnt), 0, st)
    torch.cuda.synchronize()
    uniq = [0, 3, 5, 12, 40, 63]
    assert int(b["n"].item()) == len(uniq)
    assert lst[:len(uniq)].tolist() == uniq
    assert cnt.tolist() == [3, 3]  # 0, 3, 5 borrowed; 12, 40, 63 fetched
    for bi, name in enumerate(("w13", "w2", "s13", "s2")):
        v = b[name].view(torch.uint8).reshape(64, -1).view(torch.int64)
        kk = torch.arange(v.shape[1], dtype=torch.int64, device=DEV)
        for j, e in enumerate(uniq):
            assert torch.equal(v[j], kk + ((bi << 56) | (e << 32))), (name, j, e)
    # read-only: the cache tables did not move
    assert torch.equal(ex._dc_stamp, stamp0)
    assert torch.equal(ex._dc_step, step0)
    assert torch.equal(ex._dc_slot_of, slot_of0)
    del x


@pytest.mark.parametrize("T,cap", [(64, 16), (300, 32), (5, 0)])
def test_offloaded_forward_equals_resident(T, cap):
    E = 64
    ref = synth.make_experts(E, seed=9, device="cuda")
    host = ref.to("cpu").pin()
    if cap:
        devcache.init_dev_cache(host, DEV, cap)
        devcache.dev_resolve_and_fetch(host, torch.randperm(E)[:8].to(DEV))
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16).to(DEV)
    ids = torch.stack([torch.randperm(E, generator=g)[:8] for _ in range(T)]).to(DEV)
    w = torch.rand(T, 8, generator=g)
    w = (w / w.sum(-1, keepdim=True)).to(DEV)
    want = moe.fp8_moe_forward(x, ids, w, ref.w13_weight, ref.w13_scale_inv, ref.w2_weight,
                               ref.w2_scale_inv).clone()
    got = offload.offloaded_forward(host, x, ids, w)
    moe.check_errors(DEV)
    assert torch.equal(got, want)
    if T <= 64:
        cpu = ref.to("cpu")
        o = oracle.moe_forward(x.cpu(), ids.cpu(), w.cpu(), cpu.w13_weight, cpu.w13_scale_inv,
                               cpu.w2_weight, cpu.w2_scale_inv)
        err = float((got.float().cpu() - o).abs().max() / o.abs().max())
        assert err < 1e-2, err
    # dev_cached_forward sends multi-row batches down this path
    if cap:
        got2 = devcache.dev_cached_forward(host, x, ids, w)
        assert torch.equal(got2, want)


@pytest.mark.parametrize("T", [300, 5])
def test_chunk_prefetch_equals_union_gather(T):
    """Three offloaded layers with warm caches: the cross-layer prefetch
    pipeline (offload.ChunkPrefetch) gives the same bits as gathering each
    layer's union after its router, eagerly and replayed from a CUDA graph;
    T = 5 (40 pairs for 64 experts) takes the union path inside it."""
    E, L = 64, 3
    layers = []
    for l in range(L):
        host = synth.make_experts(E, seed=20 + l, device="cuda").to("cpu").pin()
        devcache.init_dev_cache(host, DEV, 16)
        devcache.dev_resolve_and_fetch(host, torch.randperm(E)[:8 + l].to(DEV))
        layers.append(host)
    torch.cuda.synchronize()
    g = torch.Generator().manual_seed(T)
    x0 = torch.randn(T, 2048, generator=g).to(torch.bfloat16).to(DEV)
    ids = [torch.stack([torch.randperm(E, generator=g)[:8] for _ in range(T)]).to(DEV)
           for _ in range(L)]
    w = torch.rand(T, 8, generator=g)
    w = (w / w.sum(-1, keepdim=True)).to(DEV)

    def chunk(fwd, h):
        h.copy_(x0)
        for l in range(L):
            h.add_(fwd(l, h, ids[l], w))
        return h

    want = chunk(lambda l, h, i, ww: offload.offloaded_forward(layers[l], h, i, ww),
                 torch.empty_like(x0)).clone()
    c0 = [offload.gather_counters(ex) for ex in layers]
    pf = offload.ChunkPrefetch(layers, DEV)
    got = chunk(pf.forward, torch.empty_like(x0)).clone()
    moe.check_errors(DEV)
    torch.cuda.synchronize()
    assert pf._piped == (T * 8 >= 4 * E)
    assert torch.equal(got, want)
    if pf._piped:
        # the whole layer was gathered: its resident experts borrowed, the rest fetched
        for l, ex in enumerate(layers):
            c1 = offload.gather_counters(ex)
            resident = int((ex._dc_slot_of >= 0).sum())
            assert c1["gather_hits"] - c0[l]["gather_hits"] == resident
            assert c1["gather_misses"] - c0[l]["gather_misses"] == E - resident
    # captured once, replayed twice
    h = torch.empty_like(x0)
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chunk(pf.forward, h)
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        chunk(pf.forward, h)
    for _ in range(2):
        h.zero_()
        gr.replay()
        torch.cuda.synchronize()
        assert torch.equal(h, want)
    moe.check_errors(DEV)
    del gr


def test_installed_forward_runs_the_chunk_pipeline():
    """install_offload(..., chunk_prefetch=True): the experts' own forward,
    called layer by layer as the model does, runs the cross-layer pipeline
    with the union gather's bits; a layer called out of order gathers its
    union."""
    from types import SimpleNamespace

    class _Experts(synth.HostExperts):
        def forward(self, x, topk_ids, topk_weights):  # the stock forward install_offload keeps
            raise AssertionError("stock forward called")

    E, L, T = 64, 3, 300
    layers = []
    for l in range(L):
        h = synth.make_experts(E, seed=30 + l, device="cuda").to("cpu").pin()
        ex = _Experts(E, h.w13_weight, h.w2_weight, h.w13_scale_inv, h.w2_scale_inv)
        devcache.init_dev_cache(ex, DEV, 16)
        devcache.dev_resolve_and_fetch(ex, torch.randperm(E)[:8].to(DEV))
        layers.append(ex)
    g = torch.Generator().manual_seed(11)
    x0 = torch.randn(T, 2048, generator=g).to(torch.bfloat16).to(DEV)
    ids = [torch.stack([torch.randperm(E, generator=g)[:8] for _ in range(T)]).to(DEV)
           for _ in range(L)]
    w = torch.rand(T, 8, generator=g)
    w = (w / w.sum(-1, keepdim=True)).to(DEV)

    def chunk(fwd):
        h = x0.clone()
        for l in range(L):
            h.add_(fwd(l, h, ids[l], w))
        return h

    want = chunk(lambda l, h, i, ww: offload.offloaded_forward(layers[l], h, i, ww)).clone()
    want1 = offload.offloaded_forward(layers[1], x0, ids[1], w).clone()
    model = SimpleNamespace(backbone=SimpleNamespace(model=SimpleNamespace(
        layers=[SimpleNamespace(mlp=SimpleNamespace(experts=ex)) for ex in layers])))
    offload.install_offload(_Experts, model, chunk_prefetch=True)
    try:
        got = chunk(lambda l, h, i, ww: layers[l].forward(h, i, ww))
        torch.cuda.synchronize()
        pf = offload._CHAIN["pf"]
        assert pf is not None and pf._piped
        assert torch.equal(got, want)
        got1 = layers[1].forward(x0, ids[1], w)
        assert pf._next == -1
        assert torch.equal(got1, want1)
        moe.check_errors(DEV)
    finally:
        offload._CHAIN.update(layers=[], pf=None)
        for ex in layers:
            del ex._d3_chain_pos
