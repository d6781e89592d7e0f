"""GPU parity of the router and the FP8 grouped expert GEMM, through the C ABI.

* Router: expert ids bit-exact against the oracle (exactly rounded bf16
  logits, ties to the lower index); weights within 1e-5 relative.
* MoE forward: hidden states within 1e-2 relative (max|d| / max|ref|) of the
  oracle's dequantise-then-matmul path (fp32), at the single-layer
  configuration (hidden 2048, 256 experts, intermediate 512, top-8,
  N(0,0.02) weights quantised per 128x128 block, 16 tokens of N(0,1), seed 0)
  and at decode / prefill-sized batches.
* The reference's own equivalence test (bin/test_devcache.py:47-76): the
  device-cache path equals the all-resident path exactly (max|d| == 0).
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import devcache, moe, synth  # noqa: E402

DEV = torch.device("cuda:0")
TOL = 1e-2   # max|out - ref| / max|ref|, BASELINE north_star tolerance


def rel_err(got, ref):
    got = got.float().cpu()
    ref = ref.float().cpu()
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


# T <= 2: one thread-block cluster (logits in distributed shared memory);
# larger T: the general kernel (logits in the workspace, last CTA selects)
@pytest.mark.parametrize("T", [1, 2, 5, 8, 9, 16, 100, 2048])
def test_router_ids_bit_exact(T):
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    gw = (torch.randn(256, 2048, generator=g) * 0.02).to(torch.bfloat16)
    want_ids, want_w, _, ties = oracle.router_topk(x, gw, 8)
    ids, w = moe.router_topk(x.to(DEV), gw.to(DEV), 8)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids.numpy())
    np.testing.assert_allclose(w.cpu().numpy(), want_w.numpy(), rtol=1e-5, atol=1e-7)
    # repeat: the arrival counters reset themselves
    ids2, _ = moe.router_topk(x.to(DEV), gw.to(DEV), 8)
    assert torch.equal(ids2, ids)


@pytest.mark.parametrize("T", [4, 12])
def test_router_tie_break_lower_index(T):
    # identical gate rows -> identical logits; ties must resolve to lower ids
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    gw = (torch.randn(256, 2048, generator=g) * 0.02).to(torch.bfloat16)
    # three identical rows aligned with token 0 -> equal top logits for it
    row = (x[0].float().sign() * 0.05).to(torch.bfloat16)
    for e in (200, 10, 3):
        gw[e] = row
    want_ids, _, lg, _ = oracle.router_topk(x, gw, 8)
    ids, _ = moe.router_topk(x.to(DEV), gw.to(DEV), 8)
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids.numpy())
    assert ids[0, :3].tolist() == [3, 10, 200]


@pytest.mark.parametrize("T", [1, 5])
def test_router_exact_with_zeros_and_subnormals(T):
    """bf16 -> fp64 conversion by bit manipulation: zeros (both signs) and
    subnormal inputs still give the oracle's ids."""
    g = torch.Generator().manual_seed(40 + T)
    x = torch.randn(T, 2048, generator=g)
    x[:, ::7] = 0.0
    x[:, 1::13] = -0.0
    x[:, 3::11] = 1e-39            # bf16 subnormal
    gw = torch.randn(256, 2048, generator=g) * 0.02
    gw[:, ::5] = 0.0
    gw[7, 2::9] = -3e-39
    x, gw = x.to(torch.bfloat16), gw.to(torch.bfloat16)
    assert (x.float().abs() < 1.17e-38).logical_and(x.float() != 0).any()
    want_ids, want_w, _, _ = oracle.router_topk(x, gw, 8)
    ids, w = moe.router_topk(x.to(DEV), gw.to(DEV), 8)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids.numpy())
    np.testing.assert_allclose(w.cpu().numpy(), want_w.numpy(), rtol=1e-5, atol=1e-7)


def test_router_cluster_and_general_kernels_agree():
    """The same tokens routed 2 at a time (cluster kernel) and 16 at a time
    (general kernel) give identical ids and bit-identical weights."""
    g = torch.Generator().manual_seed(12)
    x = torch.randn(16, 2048, generator=g).to(torch.bfloat16).to(DEV)
    gw = (torch.randn(256, 2048, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    ids, w = moe.router_topk(x, gw, 8)
    parts = [moe.router_topk(x[i:i + 2].contiguous(), gw, 8) for i in range(0, 16, 2)]
    torch.cuda.synchronize()
    assert torch.equal(ids, torch.cat([p[0] for p in parts]))
    assert torch.equal(w, torch.cat([p[1] for p in parts]))


@pytest.fixture(scope="module")
def layer256():
    """The single-layer configuration: 256 experts, seed 0."""
    ex = synth.make_experts(256, seed=0, device="cuda", chunk=32)
    g = torch.Generator().manual_seed(0)
    gate = (torch.randn(256, 2048, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(16, 2048, generator=g).to(torch.bfloat16)
    return ex, gate, x


def test_single_layer_config(layer256):
    ex, gate, x = layer256
    ids_ref, w_ref, _, ties = oracle.router_topk(x, gate, 8)
    ids, w = moe.router_topk(x.to(DEV), gate.to(DEV), 8)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.numpy())
    out = moe.fp8_moe_forward(x.to(DEV), ids, w, ex.w13_weight, ex.w13_scale_inv,
                              ex.w2_weight, ex.w2_scale_inv)
    moe.check_errors(DEV)
    cpu = ex.to("cpu")
    ref = oracle.moe_forward(x, ids_ref, w_ref, cpu.w13_weight, cpu.w13_scale_inv,
                             cpu.w2_weight, cpu.w2_scale_inv)
    assert rel_err(out, ref) < TOL, rel_err(out, ref)
    assert torch.isfinite(out.float()).all()


def _rand_case(E, T, k, seed, ids_dtype=torch.int32, style="normal"):
    g = torch.Generator().manual_seed(seed)
    ex = synth.make_experts(E, seed=seed, device="cuda", chunk=16, style=style)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(ids_dtype)
    w = torch.rand(T, k, generator=g)
    w = w / w.sum(-1, keepdim=True)
    return ex, x, ids, w


@pytest.mark.parametrize("E,T,k,seed", [(8, 1, 8, 1), (64, 1, 8, 2), (64, 16, 8, 3),
                                        (16, 64, 4, 4), (8, 512, 8, 5), (32, 200, 8, 6)])
def test_moe_forward_matches_oracle(E, T, k, seed):
    ex, x, ids, w = _rand_case(E, T, k, seed)
    out = moe.fp8_moe_forward(x.to(DEV), ids.to(DEV), w.to(DEV), ex.w13_weight,
                              ex.w13_scale_inv, ex.w2_weight, ex.w2_scale_inv)
    moe.check_errors(DEV)
    cpu = ex.to("cpu")
    ref = oracle.moe_forward(x, ids, w, cpu.w13_weight, cpu.w13_scale_inv, cpu.w2_weight,
                             cpu.w2_scale_inv)
    assert rel_err(out, ref) < TOL, rel_err(out, ref)


@pytest.mark.parametrize("T", [2, 8])   # CUDA-core path / tensor-core path
def test_moe_forward_bf16_weights_int64_ids_and_skips(T):
    ex, x, ids, w = _rand_case(16, T, 8, 11, ids_dtype=torch.int64, style="test")
    ids[T - 1, 3] = -1
    ids[0, 0] = 16  # out of range -> skipped
    out = moe.fp8_moe_forward(x.to(DEV), ids.to(DEV), w.to(torch.bfloat16).to(DEV),
                              ex.w13_weight, ex.w13_scale_inv, ex.w2_weight, ex.w2_scale_inv)
    moe.check_errors(DEV)
    keep = (ids >= 0) & (ids < 16)
    ids_ref = torch.where(keep, ids, torch.zeros_like(ids))
    w_ref = torch.where(keep, w.to(torch.bfloat16).float(), torch.zeros_like(w))
    cpu = ex.to("cpu")
    ref = oracle.moe_forward(x, ids_ref, w_ref, cpu.w13_weight, cpu.w13_scale_inv,
                             cpu.w2_weight, cpu.w2_scale_inv)
    assert rel_err(out, ref) < TOL


def test_moe_forward_subset_invariance():
    """Results identical for all experts vs a renumbered subset
    (the gather-and-remap invariant, bin/offload.py:9-11)."""
    ex, x, ids, w = _rand_case(64, 1, 8, 21)
    full = moe.fp8_moe_forward(x.to(DEV), ids.to(DEV), w.to(DEV), ex.w13_weight,
                               ex.w13_scale_inv, ex.w2_weight, ex.w2_scale_inv).clone()
    uniq, inv = torch.unique(ids.reshape(-1), return_inverse=True)
    u = uniq.to(DEV)
    sub = moe.fp8_moe_forward(x.to(DEV), inv.reshape(ids.shape).to(DEV), w.to(DEV),
                              ex.w13_weight[u].contiguous(), ex.w13_scale_inv[u].contiguous(),
                              ex.w2_weight[u].contiguous(), ex.w2_scale_inv[u].contiguous())
    assert torch.equal(full, sub)


def test_moe_forward_graph_replay():
    ex, x, ids, w = _rand_case(32, 4, 8, 31)
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    eager = moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                                ex.w2_scale_inv).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                                  ex.w2_scale_inv)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new inputs after capture are picked up on replay
    x2 = torch.randn_like(x.float()).to(torch.bfloat16).to(DEV)
    ids2 = torch.stack([torch.randperm(32)[:8] for _ in range(4)]).to(torch.int32).to(DEV)
    xd.copy_(x2)
    idd.copy_(ids2)
    g.replay()
    want = moe.fp8_moe_forward(x2, ids2, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                               ex.w2_scale_inv)
    torch.cuda.synchronize()
    assert torch.equal(out, want)


@pytest.mark.parametrize("cap", [16, 32, 64])
def test_dev_cached_forward_equals_resident(cap):
    """bin/test_devcache.py:47-76: cache path == all-resident path, max|d| == 0."""
    E = 64
    ref = synth.make_experts(E, seed=5, device="cuda", style="test")
    host = ref.to("cpu").pin()
    devcache.init_dev_cache(host, DEV, cap)
    g = torch.Generator().manual_seed(cap)
    for step in range(40):
        x = torch.randn(1, 2048, generator=g).to(torch.bfloat16).to(DEV)
        ids = torch.randperm(E, generator=g)[:8].unsqueeze(0).to(DEV)
        w = torch.rand(1, 8, generator=g)
        w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16).to(DEV)
        want = moe.fp8_moe_forward(x, ids, w, ref.w13_weight, ref.w13_scale_inv, ref.w2_weight,
                                   ref.w2_scale_inv).clone()
        got = devcache.dev_cached_forward(host, x, ids, w)
        assert torch.equal(want, got), f"cap {cap} step {step}"
    moe.check_errors(DEV)


@pytest.mark.parametrize("cap,shared,acc,fetch_ctas", [(12, True, True, 32), (8, False, False, 32),
                                                      (24, True, False, 5), (64, True, True, 148)])
def test_fetch_gate_up_overlap_matches_separate_launches(cap, shared, acc, fetch_ctas):
    """d3_resolve_fetch_moe (fetch + gate/up in one launch, each fetched
    expert's gate/up after its bytes land) against d3_resolve_fetch followed
    by the decode MoE call over the cache: the same slot tables and
    bit-identical outputs, step after step (misses, hits, evictions)."""
    E, H, I = 64, 2048, 512
    ref = synth.make_experts(E, seed=9, device="cuda", style="test")
    a, b = ref.to("cpu").pin(), ref.to("cpu").pin()
    devcache.init_dev_cache(a, DEV, cap)
    devcache.init_dev_cache(b, DEV, cap)
    sh = tuple(t.to(DEV) if t is not None else None for t in _shared(H, I, seed=cap)) \
        if shared else None
    g = torch.Generator().manual_seed(100 + cap)
    old = devcache.OVERLAP_FETCH_CTAS
    devcache.OVERLAP_FETCH_CTAS = fetch_ctas
    try:
        for step in range(30):
            x = torch.randn(1, H, generator=g).to(torch.bfloat16).to(DEV)
            ids = torch.randperm(E if step % 3 else 16, generator=g)[:8].unsqueeze(0).to(DEV)
            w = torch.rand(1, 8, generator=g).to(DEV)
            base = torch.randn(1, H, generator=g).to(torch.bfloat16).to(DEV)
            out_a, out_b = base.clone(), base.clone()
            devcache.dev_resolve_fetch_moe(a, ids, x, w, out=out_a, accumulate=acc, shared=sh)
            slots = devcache.dev_resolve_and_fetch(b, ids)
            moe.fp8_moe_forward(x, slots.reshape(1, 8), w, b._dc_w13, b._dc_s13, b._dc_w2,
                                b._dc_s2, out=out_b, accumulate=acc, shared=sh)
            torch.cuda.synchronize()
            assert torch.equal(a._dc_out, b._dc_out), f"step {step}"
            assert torch.equal(a._dc_slot_expert, b._dc_slot_expert), f"step {step}"
            assert torch.equal(out_a, out_b), f"step {step}"
    finally:
        devcache.OVERLAP_FETCH_CTAS = old
    moe.check_errors(DEV)
    assert torch.equal(a._dc_w13, b._dc_w13) and torch.equal(a._dc_s2, b._dc_s2)


def test_l2_warm_window_changes_nothing_but_timing():
    """d3_resolve_fetch_moe_l2warm (the fused decode call with L2 warm
    windows: one, two, ragged sizes) gives the slots and bits of
    d3_resolve_fetch_moe, step after step; the windows' bytes are untouched."""
    E, H, I = 64, 2048, 512
    ref = synth.make_experts(E, seed=13, device="cuda", style="test")
    a, b = ref.to("cpu").pin(), ref.to("cpu").pin()
    devcache.init_dev_cache(a, DEV, 12)
    devcache.init_dev_cache(b, DEV, 12)
    warm = torch.randn(3 << 20, device=DEV).to(torch.bfloat16)   # 6 MiB of "next-layer weights"
    gate = torch.randn(256, 2048, device=DEV).to(torch.bfloat16)  # a second window (1 MiB)
    warm0, gate0 = warm.clone(), gate.clone()
    g = torch.Generator().manual_seed(77)
    for step in range(20):
        x = torch.randn(1, H, generator=g).to(torch.bfloat16).to(DEV)
        ids = torch.randperm(E, generator=g)[:8].unsqueeze(0).to(DEV)
        w = torch.rand(1, 8, generator=g).to(DEV)
        nb = None if step % 2 else (step * 65537) % (6 << 20)   # whole window / ragged sizes
        if step % 3 == 2:   # two windows
            out_a = devcache.dev_resolve_fetch_moe(a, ids, x, w, l2_warm=[gate, warm],
                                                   l2_warm_bytes=[None, nb])
        else:
            out_a = devcache.dev_resolve_fetch_moe(a, ids, x, w, l2_warm=warm, l2_warm_bytes=nb)
        out_b = devcache.dev_resolve_fetch_moe(b, ids, x, w)
        torch.cuda.synchronize()
        assert torch.equal(a._dc_out, b._dc_out), f"step {step}"
        assert torch.equal(out_a, out_b), f"step {step}"
    moe.check_errors(DEV)
    assert torch.equal(warm, warm0) and torch.equal(gate, gate0)


@pytest.mark.parametrize("T", [1, 5])   # CUDA-core path / tensor-core path
def test_moe_forward_accumulate_into_input(T):
    """accumulate=True with out aliasing x: h <- h + moe(h) (the residual add)."""
    ex, x, ids, w = _rand_case(16, T, 8, 41)
    xd = x.to(DEV)
    plain = moe.fp8_moe_forward(xd, ids.to(DEV), w.to(DEV), ex.w13_weight, ex.w13_scale_inv,
                                ex.w2_weight, ex.w2_scale_inv).clone()
    h = xd.clone()
    moe.fp8_moe_forward(h, ids.to(DEV), w.to(DEV), ex.w13_weight, ex.w13_scale_inv,
                        ex.w2_weight, ex.w2_scale_inv, out=h, accumulate=True)
    moe.check_errors(DEV)
    want = xd.float() + plain.float()
    assert rel_err(h, want) < 1e-2


@pytest.mark.parametrize("T", [1, 2, 4])
def test_moe_small_batch_paths_agree(T, monkeypatch):
    """Decode-sized batches run on the CUDA cores (GEMV, fp32 activations);
    forced onto the tensor-core path (D3_GEMV_MAX_PAIRS=0) the same call must
    agree with it and with the oracle within the tolerance."""
    ex, x, ids, w = _rand_case(64, T, 8, 50 + T)
    args = (x.to(DEV), ids.to(DEV), w.to(DEV), ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
            ex.w2_scale_inv)
    gemv = moe.fp8_moe_forward(*args).clone()
    monkeypatch.setenv("D3_GEMV_MAX_PAIRS", "0")
    gemm = moe.fp8_moe_forward(*args).clone()
    moe.check_errors(DEV)
    cpu = ex.to("cpu")
    ref = oracle.moe_forward(x, ids, w, cpu.w13_weight, cpu.w13_scale_inv, cpu.w2_weight,
                             cpu.w2_scale_inv)
    assert rel_err(gemv, ref) < TOL, rel_err(gemv, ref)
    assert rel_err(gemm, ref) < TOL, rel_err(gemm, ref)
    assert rel_err(gemv, gemm) < TOL
    # the fp32-activation path sits closer to the fp32 oracle
    assert rel_err(gemv, ref) <= rel_err(gemm, ref) * 1.5 + 1e-3


@pytest.mark.parametrize("E,T,k", [(8, 512, 8), (64, 16, 8), (68, 1, 8), (68, 2, 8)])
def test_moe_forward_deterministic_with_fresh_inputs(E, T, k):
    """Repeated calls, each right after fresh host->device copies of its inputs,
    give bit-identical results (no launch of a call may start before the
    caller's preceding stream work)."""
    ex, x, ids, w = _rand_case(E, T, k, 77)
    outs = []
    for _ in range(3):
        xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
        out = moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                                  ex.w2_scale_inv)
        outs.append(out.clone())
        del xd, idd, wd
    torch.cuda.synchronize()
    moe.check_errors(DEV)
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert torch.isfinite(outs[0].float()).all()


def _shared(H=2048, I=512, seed=3, gated=True):
    g = torch.Generator().manual_seed(seed)
    sw13 = (torch.randn(2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    sw2 = (torch.randn(H, I, generator=g) * 0.02).to(torch.bfloat16)
    sg = (torch.randn(H, generator=g) * 0.02).to(torch.bfloat16) if gated else None
    return sw13, sw2, sg


@pytest.mark.parametrize("T,gated,acc", [(1, True, False), (2, True, True), (4, False, False),
                                         (16, True, False), (16, True, True)])
def test_moe_forward_with_shared_expert(T, gated, acc):
    """Routed experts + Drama-3's gated shared expert: fused into the two
    decode launches (T * 8 <= 32), two plain bf16 GEMMs beside the routed
    path above that; both against the oracle."""
    ex, x, ids, w = _rand_case(64, T, 8, 60 + T)
    sw13, sw2, sg = _shared(gated=gated)
    xd = x.to(DEV)
    out = xd.clone() if acc else None
    shared = (sw13.to(DEV), sw2.to(DEV), sg.to(DEV) if sg is not None else None)
    got = moe.fp8_moe_forward(xd, ids.to(DEV), w.to(DEV), ex.w13_weight, ex.w13_scale_inv,
                              ex.w2_weight, ex.w2_scale_inv, out=out, accumulate=acc,
                              shared=shared)
    moe.check_errors(DEV)
    cpu = ex.to("cpu")
    ref = oracle.moe_forward(x, ids, w, cpu.w13_weight, cpu.w13_scale_inv, cpu.w2_weight,
                             cpu.w2_scale_inv)
    ref = ref + oracle.shared_expert_forward(x, sw13, sw2, sg)
    if acc:
        ref = ref + x.float()
    assert rel_err(got, ref) < TOL, rel_err(got, ref)


def test_shared_expert_fused_entry_rejects_large_batch():
    from drama3_offloading_b200 import _lib
    ex, x, ids, w = _rand_case(16, 8, 8, 70)     # 64 pairs: not a decode batch
    sw13, sw2, sg = [t.to(DEV) for t in _shared(seed=4)]
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    out = torch.empty_like(xd)
    need = moe.workspace_bytes(8, 8, 16, 2048, 512)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    P = _lib.ptr
    with pytest.raises(_lib.D3Error) as ei:
        _lib.call("d3_moe_fp8_forward_shared", P(xd), P(idd), 4, P(wd), 1, 8, 8,
                  P(ex.w13_weight), P(ex.w13_scale_inv), P(ex.w2_weight), P(ex.w2_scale_inv),
                  16, 2048, 512, P(sw13), P(sw2), P(sg), P(out), 0, P(moe.error_word(DEV)),
                  P(ws), ws.numel(), _lib.stream_ptr())
    assert ei.value.status == -5   # D3_ERR_UNSUPPORTED
