"""GPU parity of the expert path on sparse batches -- a few routed pairs per
expert, most of them on the tensor-core path -- through the C ABI, against the
oracle's dequantise-then-matmul restatement (max|d| / max|ref| < 1e-2).

Shapes: the expert-parallel receive buffer (one slot per row, most rows empty:
id -1), experts with many more tokens than others, top-k batches with the
combine, int64 ids, bf16 weights, skipped ids, the residual add into the
input, repeat determinism, and independence of the expert numbering.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import moe, synth  # noqa: E402

DEV = torch.device("cuda:0")
TOL = 1e-2


def rel_err(got, ref):
    got = got.float().cpu()
    ref = ref.float().cpu()
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def _ref(x, ids, w, ex):
    keep = ids >= 0
    ids_r = torch.where(keep, ids, torch.zeros_like(ids)).to(torch.int64)
    w_r = torch.where(keep, w.float(), torch.zeros_like(w.float()))
    cpu = ex.to("cpu")
    return oracle.moe_forward(x, ids_r, w_r, cpu.w13_weight, cpu.w13_scale_inv, cpu.w2_weight,
                              cpu.w2_scale_inv)


def _ep_case(E, rows, valid, seed, ids_dtype=torch.int32):
    g = torch.Generator().manual_seed(seed)
    ex = synth.make_experts(E, seed=seed, device="cuda", chunk=16)
    x = torch.randn(rows, 2048, generator=g).to(torch.bfloat16)
    ids = torch.full((rows, 1), -1, dtype=ids_dtype)
    pos = torch.randperm(rows, generator=g)[:valid]
    ids[pos, 0] = torch.randint(0, E, (valid,), generator=g).to(ids_dtype)
    w = torch.ones(rows, 1)
    return ex, x, ids, w


def _run(ex, x, ids, w, **kw):
    out = moe.fp8_moe_forward(x.to(DEV), ids.to(DEV), w.to(DEV), ex.w13_weight,
                              ex.w13_scale_inv, ex.w2_weight, ex.w2_scale_inv, **kw)
    moe.check_errors(DEV)
    return out


@pytest.mark.parametrize("E,rows,valid", [(32, 512, 64), (64, 512, 128), (16, 96, 96),
                                          (4, 200, 200)])
def test_sparse_ep_receive_buffer(E, rows, valid):
    """One slot per row, most rows empty (-1): the expert-parallel layout."""
    ex, x, ids, w = _ep_case(E, rows, valid, seed=E + rows)
    out = _run(ex, x, ids, w).clone()
    ref = _ref(x, ids, w, ex)
    assert rel_err(out, ref) < TOL, rel_err(out, ref)
    empty = (ids[:, 0] < 0).nonzero().flatten()
    assert torch.count_nonzero(out[empty.to(DEV)]) == 0   # empty rows are zero


@pytest.mark.parametrize("T,k", [(16, 8), (5, 8), (40, 4)])
def test_sparse_topk_combine(T, k):
    g = torch.Generator().manual_seed(T * 10 + k)
    E = 64
    ex = synth.make_experts(E, seed=7, device="cuda", chunk=16)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    w = w / w.sum(-1, keepdim=True)
    out = _run(ex, x, ids, w)
    assert rel_err(out, _ref(x, ids, w, ex)) < TOL


def test_sparse_int64_bf16_weights_skips_accumulate():
    E, T, k = 16, 12, 8
    g = torch.Generator().manual_seed(5)
    ex = synth.make_experts(E, seed=5, device="cuda", chunk=16, style="test")
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int64)
    ids[3, 2] = -1
    ids[7, 0] = E + 4                      # out of range: skipped
    w = torch.rand(T, k, generator=g).to(torch.bfloat16)
    xd = x.to(DEV)
    h = xd.clone()
    moe.fp8_moe_forward(h, ids.to(DEV), w.to(DEV), ex.w13_weight, ex.w13_scale_inv,
                        ex.w2_weight, ex.w2_scale_inv, out=h, accumulate=True)
    moe.check_errors(DEV)
    ids_r = torch.where(ids < E, ids, torch.full_like(ids, -1))
    want = x.float() + _ref(x, ids_r, w, ex)
    assert rel_err(h, want) < TOL


def test_sparse_deterministic_and_numbering_invariant():
    E, rows, valid = 48, 256, 200
    ex, x, ids, w = _ep_case(E, rows, valid, seed=9)
    outs = [_run(ex, x, ids, w).clone() for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    # renumber the experts in use (a compact subset, reversed order)
    used = torch.unique(ids[ids >= 0])
    perm = torch.full((E,), -1, dtype=torch.int64)
    perm[used] = torch.arange(len(used) - 1, -1, -1)
    sub_ids = torch.where(ids >= 0, perm[ids.clamp_min(0).long()], torch.full_like(ids, -1).long())
    src = used.flip(0).to(DEV)
    sub = moe.fp8_moe_forward(x.to(DEV), sub_ids.to(torch.int32).to(DEV), w.to(DEV),
                              ex.w13_weight[src].contiguous(), ex.w13_scale_inv[src].contiguous(),
                              ex.w2_weight[src].contiguous(), ex.w2_scale_inv[src].contiguous())
    moe.check_errors(DEV)
    assert torch.equal(outs[0], sub)
