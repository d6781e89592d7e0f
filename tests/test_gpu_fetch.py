"""GPU parity of the slot allocator and the expert fetch, through the C ABI.

Checked against the reference's own kernels (golden fixtures from the
interpreted Triton ``_resolve_slots``/``_fetch_experts``) and the CPU oracle:
slot assignments, fetch job lists and every fetched byte must match exactly.
Mirrors the reference's bin/test_devcache.py (capacities 16/32/64 of 64
experts, 40 steps, CUDA-graph capture replaying DYNAMIC) and
bin/bench_hostread.py's self-identifying byte pattern and njobs-shrink check.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import _lib, devcache, synth  # noqa: E402

DEV = torch.device("cuda:0")
CASES = ["small_dups", "k_gt_c", "randperm_c16", "randperm_c32", "randperm_c64",
         "zipf_c51", "zipf_c68", "global_pool"]


def _resolve(ids, tabs, out, fs, fe, nm, C, E):
    _lib.call("d3_resolve_slots", _lib.ptr(ids), ids.element_size(), ids.numel(),
              _lib.ptr(tabs["slot_of"]), E, _lib.ptr(tabs["slot_expert"]),
              _lib.ptr(tabs["stamp"]), C, _lib.ptr(out), _lib.ptr(fs), _lib.ptr(fe),
              _lib.ptr(nm), _lib.ptr(tabs["step"]), _lib.stream_ptr())


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("id_dtype", [torch.int32, torch.int64])
def test_resolve_slots_matches_reference(golden, case, id_dtype):
    g = lambda k: golden[f"{case}/{k}"]
    E, C = int(g("E")), int(g("C"))
    ids_all = torch.from_numpy(g("ids")).to(id_dtype).to(DEV)
    K = ids_all.shape[1]
    tabs = {"slot_of": torch.full((E,), -1, dtype=torch.int32, device=DEV),
            "slot_expert": torch.full((C,), -1, dtype=torch.int32, device=DEV),
            "stamp": -torch.arange(C, 0, -1, dtype=torch.int64, device=DEV),
            "step": torch.zeros(1, dtype=torch.int64, device=DEV)}
    out = torch.zeros(K, dtype=torch.int32, device=DEV)
    fs = torch.zeros(K, dtype=torch.int32, device=DEV)
    fe = torch.zeros(K, dtype=torch.int32, device=DEV)
    nm = torch.zeros(1, dtype=torch.int32, device=DEV)
    outs, fss, fes, nms = [], [], [], []
    for i in range(ids_all.shape[0]):
        _resolve(ids_all[i].contiguous(), tabs, out, fs, fe, nm, C, E)
        outs.append(out.clone()); fss.append(fs.clone()); fes.append(fe.clone())
        nms.append(nm.clone())
    torch.cuda.synchronize()
    for i in range(ids_all.shape[0]):
        n = int(nms[i].item())
        assert n == int(g("nmiss")[i]), f"call {i}"
        np.testing.assert_array_equal(outs[i].cpu().numpy(), g("out")[i])
        np.testing.assert_array_equal(fss[i].cpu().numpy()[:n], g("fslot")[i][:n])
        np.testing.assert_array_equal(fes[i].cpu().numpy()[:n], g("fexp")[i][:n])
    np.testing.assert_array_equal(tabs["slot_of"].cpu().numpy(), g("final_slot_of"))
    np.testing.assert_array_equal(tabs["slot_expert"].cpu().numpy(), g("final_slot_expert"))
    np.testing.assert_array_equal(tabs["stamp"].cpu().numpy(), g("final_stamp"))
    np.testing.assert_array_equal(tabs["step"].cpu().numpy(), g("final_step"))


@pytest.mark.parametrize("offset", [2**31 - 24, 2**40])
def test_resolve_slots_large_stamps(golden, offset):
    """Stamps and steps past the int32 range take the allocator's 64-bit
    victim search: starting 24 calls below 2^31 the first calls run the
    32-bit search and the later ones cross over mid-sequence; starting at
    2^40 every call runs the 64-bit one.  Slots, jobs and final tables must
    equal the oracle's, as at small stamps."""
    g = lambda k: golden[f"zipf_c68/{k}"]
    E, C = int(g("E")), int(g("C"))
    ids_all = torch.from_numpy(g("ids")).to(torch.int32).to(DEV)
    K = ids_all.shape[1]
    tab = oracle.init_tables(E, C)
    tab.stamp += offset
    tab.step += offset
    tabs = {"slot_of": torch.from_numpy(tab.slot_of.copy()).to(DEV),
            "slot_expert": torch.from_numpy(tab.slot_expert.copy()).to(DEV),
            "stamp": torch.from_numpy(tab.stamp.copy()).to(DEV),
            "step": torch.from_numpy(tab.step.copy()).to(DEV)}
    out = torch.zeros(K, dtype=torch.int32, device=DEV)
    fs = torch.zeros(K, dtype=torch.int32, device=DEV)
    fe = torch.zeros(K, dtype=torch.int32, device=DEV)
    nm = torch.zeros(1, dtype=torch.int32, device=DEV)
    for i in range(ids_all.shape[0]):
        _resolve(ids_all[i].contiguous(), tabs, out, fs, fe, nm, C, E)
        want, wfs, wfe, n = oracle.resolve(tab, ids_all[i].cpu().numpy())
        torch.cuda.synchronize()
        assert int(nm.item()) == n, f"call {i}"
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        np.testing.assert_array_equal(fs.cpu().numpy()[:n], wfs)
        np.testing.assert_array_equal(fe.cpu().numpy()[:n], wfe)
    np.testing.assert_array_equal(tabs["slot_of"].cpu().numpy(), tab.slot_of)
    np.testing.assert_array_equal(tabs["slot_expert"].cpu().numpy(), tab.slot_expert)
    np.testing.assert_array_equal(tabs["stamp"].cpu().numpy(), tab.stamp)
    np.testing.assert_array_equal(tabs["step"].cpu().numpy(), tab.step)


@pytest.fixture(scope="module")
def pattern_host():
    """64 experts at the real dims, self-identifying bytes, pinned."""
    return synth.pattern_experts(64)


def _check_cache_bytes(ex, host):
    """Every occupied slot holds its expert's exact bytes in all four buffers."""
    se = ex._dc_slot_expert.cpu().tolist()
    caches = [ex._dc_w13, ex._dc_w2, ex._dc_s13, ex._dc_s2]
    for b, cache in enumerate(caches):
        v = cache.view(torch.uint8).reshape(cache.shape[0], -1).view(torch.int64)
        n64 = v.shape[1]
        k = torch.arange(n64, dtype=torch.int64, device=DEV)
        for s, e in enumerate(se):
            if e < 0:
                continue
            want = k + ((b << 56) | (e << 32))
            assert torch.equal(v[s], want), f"buffer {b} slot {s} expert {e}"


@pytest.mark.parametrize("backend", ["b200", "cpp"])
@pytest.mark.parametrize("cap", [16, 32, 64])
def test_resolve_fetch_lru_bytes(pattern_host, backend, cap):
    ex = synth.HostExperts(64, pattern_host.w13_weight, pattern_host.w2_weight,
                           pattern_host.w13_scale_inv, pattern_host.w2_scale_inv)
    old = devcache.FETCH_BACKEND
    devcache.FETCH_BACKEND = backend
    try:
        devcache.init_dev_cache(ex, DEV, cap, policy="lru")
        tab = oracle.init_tables(64, cap)
        gen = torch.Generator().manual_seed(cap)
        hits = misses = 0
        for step in range(40):
            ids = torch.randperm(64, generator=gen)[:8]
            slots = devcache.dev_resolve_and_fetch(ex, ids.to(DEV).unsqueeze(0))
            want, _, _, n = oracle.resolve(tab, ids.numpy())
            np.testing.assert_array_equal(slots.cpu().numpy(), want, err_msg=f"step {step}")
            assert int(ex._dc_nmiss.item()) == n
            hits += 8 - n
            misses += n
            if step % 13 == 0 or step == 39:
                _check_cache_bytes(ex, pattern_host)
        np.testing.assert_array_equal(ex._dc_slot_of.cpu().numpy(), tab.slot_of)
        np.testing.assert_array_equal(ex._dc_stamp.cpu().numpy(), tab.stamp)
        if backend == "b200":
            st = devcache.stats(ex)
            assert st == {"calls": 40, "hits": hits, "misses": misses,
                          "bytes_fetched": misses * devcache.EXPERT_BYTES}
    finally:
        devcache.FETCH_BACKEND = old


def test_resolve_fetch_lfu_bytes(pattern_host):
    ex = synth.HostExperts(64, pattern_host.w13_weight, pattern_host.w2_weight,
                           pattern_host.w13_scale_inv, pattern_host.w2_scale_inv)
    devcache.init_dev_cache(ex, DEV, 20, policy="lfu")
    tab = oracle.init_tables(64, 20)
    from drama3_offloading_b200.trace import zipf_trace
    tr = zipf_trace(steps=60, layers=1, experts=64)
    for step in range(60):
        ids = torch.from_numpy(tr[step, 0].astype(np.int64))
        slots = devcache.dev_resolve_and_fetch(ex, ids.to(DEV))
        want, _, _, n = oracle.resolve_lfu(tab, ids.numpy())
        np.testing.assert_array_equal(slots.cpu().numpy(), want, err_msg=f"step {step}")
    np.testing.assert_array_equal(ex._dc_freq.cpu().numpy(), tab.freq)
    np.testing.assert_array_equal(ex._dc_slot_expert.cpu().numpy(), tab.slot_expert)
    _check_cache_bytes(ex, pattern_host)


def test_capture_replays_dynamic(pattern_host):
    """bin/test_devcache.py:80-133: ids changed after capture must be served."""
    ex = synth.HostExperts(64, pattern_host.w13_weight, pattern_host.w2_weight,
                           pattern_host.w13_scale_inv, pattern_host.w2_scale_inv)
    devcache.init_dev_cache(ex, DEV, 32)
    g = torch.Generator().manual_seed(7)
    ids_warm = torch.randperm(64, generator=g)[:8].to(DEV)
    ids_cap = torch.randperm(64, generator=g)[:8].to(DEV)
    ids_rep = torch.randperm(64, generator=g)[:8].to(DEV)
    live = ids_warm.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            devcache.dev_resolve_and_fetch(ex, live)
    torch.cuda.current_stream().wait_stream(s)
    live.copy_(ids_cap)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = devcache.dev_resolve_and_fetch(ex, live)
    live.copy_(ids_rep)
    graph.replay()
    torch.cuda.synchronize()
    occupant = ex._dc_slot_expert[out.to(torch.int64)]
    assert torch.equal(occupant, ids_rep.to(torch.int32)), "replay FROZEN or WRONG"
    _check_cache_bytes(ex, pattern_host)
    # replay again with a second id set: the step counter advances on device
    step_before = int(ex._dc_step.item())
    live.copy_(torch.randperm(64, generator=g)[:8].to(DEV))
    graph.replay()
    torch.cuda.synchronize()
    assert int(ex._dc_step.item()) == step_before + 1
    assert torch.equal(ex._dc_slot_expert[out.to(torch.int64)], live.to(torch.int32))
    _check_cache_bytes(ex, pattern_host)


def test_fetch_experts_golden_and_njobs(golden):
    """d3_fetch_experts (fetch_experts.cu replacement) reproduces the reference
    fixture and honours a device job count below the grid's job count."""
    host = torch.from_numpy(golden["fetch/host"]).pin_memory()
    E, elems = host.shape
    C = golden["fetch/cache_after"].shape[0]
    cache = torch.full((C, elems), int(golden["fetch/fill"]), dtype=torch.uint8, device=DEV)
    dptr = ctypes.c_void_p(0)
    _lib.call("d3_device_ptr_of", ctypes.c_void_p(host.data_ptr()),
              ctypes.c_size_t(host.numel()), ctypes.byref(dptr))
    fexp = torch.from_numpy(golden["fetch/fexp"]).to(DEV)
    fslot = torch.from_numpy(golden["fetch/fslot"]).to(DEV)
    nm = torch.from_numpy(golden["fetch/nmiss"]).to(DEV)
    _lib.call("d3_fetch_experts", dptr, _lib.ptr(cache), _lib.ptr(fexp), _lib.ptr(fslot),
              _lib.ptr(nm), elems, fexp.numel(), 2, 256, _lib.stream_ptr())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.cpu().numpy(), golden["fetch/cache_after"])


def test_pageable_host_rejected():
    t = torch.zeros(1 << 16, dtype=torch.uint8)  # pageable
    with pytest.raises(_lib.D3Error) as ei:
        out = ctypes.c_void_p(0)
        _lib.call("d3_device_ptr_of", ctypes.c_void_p(t.data_ptr()), ctypes.c_size_t(t.numel()),
                  ctypes.byref(out))
    assert ei.value.status == -2


def test_out_of_range_id_not_fetched(pattern_host):
    ex = synth.HostExperts(64, pattern_host.w13_weight, pattern_host.w2_weight,
                           pattern_host.w13_scale_inv, pattern_host.w2_scale_inv)
    devcache.init_dev_cache(ex, DEV, 8)
    ids = torch.tensor([3, 64, 5, -1, 7], dtype=torch.int32, device=DEV)
    slots = devcache.dev_resolve_and_fetch(ex, ids).cpu().tolist()
    assert slots[1] == -1 and slots[3] == -1
    assert int(ex._dc_nmiss.item()) == 3
    _check_cache_bytes(ex, pattern_host)


def test_misaligned_rejected():
    cache = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    host = torch.zeros(4096, dtype=torch.uint8).pin_memory()
    z = torch.zeros(1, dtype=torch.int32, device=DEV)
    with pytest.raises(_lib.D3Error) as ei:
        _lib.call("d3_fetch_experts", ctypes.c_void_p(host.data_ptr()), _lib.ptr(cache),
                  _lib.ptr(z), _lib.ptr(z), _lib.ptr(z), 24, 1, 1, 256, _lib.stream_ptr())
    assert ei.value.status == -3
