"""The one-launch expert call (moe_fused_kernel: route, gate/up GEMM, SwiGLU,
down GEMM and combine in one cooperative launch with grid-wide phase
barriers) against the separate launches (D3_MOE_FUSED=0), through the C ABI:
bit-identical outputs at the expert-parallel shapes (the N = 8 rank's 512
received rows of which 64 are valid over 32 local experts; the 1-GPU batch
of 64 tokens over 256 experts), the single-layer configuration, the BN = 64
tiles, int64 ids with skipped pairs, the residual accumulate, repeated calls
(the grid counter returns to zero) and CUDA-graph replay; and within the
BASELINE tolerance of the oracle."""
import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import moe, synth  # noqa: E402

DEV = torch.device("cuda:0")


def _ep_rows(N, seed):
    """One rank's received rows at the N-GPU expert-parallel shape."""
    rng = np.random.default_rng(seed)
    epr, T_local = 256 // N, 64 // N
    cap = T_local * 8
    ids = np.full(N * cap, -1, np.int32)
    for s in range(N):
        toks = np.stack([rng.permutation(256)[:8] for _ in range(T_local)])
        mine = toks[toks // epr == 0] % epr
        ids[s * cap: s * cap + len(mine)] = mine
    return epr, torch.from_numpy(ids).view(-1, 1)


def _cases():
    g = torch.Generator().manual_seed(5)
    out = []
    # expert-parallel rank at N = 8: 512 rows, 64 valid, 32 experts, topk 1
    epr, ids = _ep_rows(8, 1)
    out.append(("ep8", epr, torch.randn(ids.shape[0], 2048, generator=g), ids,
                torch.ones(ids.shape[0], 1)))
    # 1-GPU expert-parallel batch: 64 tokens, uniform top-8 over 256 experts
    ids = torch.stack([torch.randperm(256, generator=g)[:8] for _ in range(64)]).to(torch.int32)
    w = torch.rand(64, 8, generator=g)
    out.append(("ep1", 256, torch.randn(64, 2048, generator=g), ids, w / w.sum(-1, keepdim=True)))
    # BN = 64 tiles: 256 tokens over 8 experts, int64 ids with skipped pairs
    ids = torch.stack([torch.randperm(8, generator=g)[:8] for _ in range(256)]).to(torch.int64)
    ids[3, 2] = -1
    ids[100, 7] = 8
    out.append(("bn64", 8, torch.randn(256, 2048, generator=g), ids, torch.rand(256, 8, generator=g)))
    return out


@pytest.fixture(scope="module")
def cases():
    res = []
    for name, E, x, ids, w in _cases():
        ex = synth.make_experts(E, seed=len(res) + 3, device="cuda", chunk=16)
        res.append((name, ex, x.to(torch.bfloat16), ids, w))
    return res


def _run(monkeypatch, fused, ex, x, ids, w, out=None, accumulate=False):
    monkeypatch.setenv("D3_MOE_FUSED", "1" if fused else "0")
    y = moe.fp8_moe_forward(x, ids, w, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv, out=out, accumulate=accumulate)
    torch.cuda.synchronize()
    moe.check_errors(DEV)
    return y.clone()


@pytest.mark.parametrize("k", range(3))
def test_fused_equals_separate_launches(monkeypatch, cases, k):
    name, ex, x, ids, w = cases[k]
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    sep = _run(monkeypatch, False, ex, xd, idd, wd)
    fus = _run(monkeypatch, True, ex, xd, idd, wd)
    again = _run(monkeypatch, True, ex, xd, idd, wd)     # the grid counter came back to zero
    assert torch.equal(fus, sep), float((fus.float() - sep.float()).abs().max())
    assert torch.equal(again, fus)
    cpu = ex.to("cpu")
    keep = (ids >= 0) & (ids < ex.num_experts)
    ref = oracle.moe_forward(x, torch.where(keep, ids, torch.zeros_like(ids)),
                             torch.where(keep, w, torch.zeros_like(w)), cpu.w13_weight,
                             cpu.w13_scale_inv, cpu.w2_weight, cpu.w2_scale_inv)
    valid = keep.any(-1)
    err = float((fus.float().cpu()[valid] - ref[valid]).abs().max() / ref[valid].abs().max())
    print(f"\n{name}: rel err vs oracle {err:.2e}")
    assert err < 1e-2


def test_fused_residual_accumulate_in_place(monkeypatch, cases):
    """out aliasing x with accumulate (the MoE block's residual add)."""
    name, ex, x, ids, w = cases[1]
    h0 = x.to(DEV)
    a = h0.clone()
    _run(monkeypatch, False, ex, a, ids.to(DEV), w.to(DEV), out=a, accumulate=True)
    b = h0.clone()
    _run(monkeypatch, True, ex, b, ids.to(DEV), w.to(DEV), out=b, accumulate=True)
    assert torch.equal(a, b)


def test_fused_graph_replay(monkeypatch, cases):
    monkeypatch.setenv("D3_MOE_FUSED", "1")
    name, ex, x, ids, w = cases[0]
    xd, idd, wd = x.to(DEV), ids.to(DEV), w.to(DEV)
    eager = _run(monkeypatch, True, ex, xd, idd, wd)
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        moe.fp8_moe_forward(xd, idd, wd, ex.w13_weight, ex.w13_scale_inv, ex.w2_weight,
                            ex.w2_scale_inv, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    moe.check_errors(DEV)
