"""Expert-parallel dispatch/combine kernels on one GPU (n_ranks simulated)
against the torch restatement, and -- when two GPUs are visible -- the
2-rank NCCL expert-parallel layer against the single-GPU MoE forward."""
import os
import socket
import sys

import pytest
import torch

from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import ep_reference as ref  # noqa: E402
from drama3_offloading_b200 import _lib, moe, synth  # noqa: E402

DEV = torch.device("cuda:0")


@pytest.mark.parametrize("n_ranks,T,k,cap", [(4, 16, 8, 128), (2, 3, 8, 24), (8, 8, 8, 5)])
def test_dispatch_pack_and_combine(n_ranks, T, k, cap):
    E, H = 256, 2048
    epr = E // n_ranks
    g = torch.Generator().manual_seed(T * 7 + n_ranks)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    ids[0, 0] = -1  # skipped pair
    w = torch.rand(T, k, generator=g)
    want_x, want_eid, want_src = ref.pack(x, ids, n_ranks, epr, cap)
    xd, idd = x.to(DEV), ids.to(DEV)
    send_x = torch.zeros(n_ranks * cap, H, dtype=torch.bfloat16, device=DEV)
    send_eid = torch.zeros(n_ranks * cap, dtype=torch.int32, device=DEV)
    src = torch.zeros(T, k, dtype=torch.int32, device=DEV)
    ovf = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.call("d3_ep_dispatch_pack", _lib.ptr(xd), _lib.ptr(idd), T, k, H, n_ranks, epr, cap,
              _lib.ptr(send_x), _lib.ptr(send_eid), _lib.ptr(src), _lib.ptr(ovf),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(send_eid.cpu(), want_eid)
    assert torch.equal(src.cpu(), want_src)
    used = want_eid >= 0
    assert torch.equal(send_x.cpu()[used], want_x[used])
    # capacity overflow is counted, not written out of bounds
    expected_overflow = int((ids.reshape(-1) >= 0).sum()) - int(used.sum())
    assert int(ovf.item()) == expected_overflow
    # combine of arbitrary returned rows
    ret = torch.randn(n_ranks * cap, H, generator=g).to(torch.bfloat16)
    out = torch.zeros(T, H, dtype=torch.bfloat16, device=DEV)
    ret_d, w_d = ret.to(DEV), w.to(DEV)   # kept alive until the kernel has run
    _lib.call("d3_ep_combine", _lib.ptr(ret_d), _lib.ptr(src), _lib.ptr(w_d), 1, T,
              k, H, _lib.ptr(out), 0, _lib.stream_ptr())
    torch.cuda.synchronize()
    want = ref.combine(ret, want_src, w)
    assert torch.allclose(out.float().cpu(), want, atol=2e-2, rtol=1e-2)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        from drama3_offloading_b200.ep import ExpertParallelMoE
        from drama3_offloading_b200.trace import uniform_trace
        dev = torch.device("cuda", rank)
        tr = uniform_trace(steps=4, tokens=16, layers=2, experts=256, k=8)
        m = ExpertParallelMoE(layers=2, global_batch=16, rank=rank, world=world,
                              device=dev, trace=tr)
        h0 = m.h.clone()
        m.step()
        torch.cuda.synchronize()
        hs = [torch.zeros_like(m.h) for _ in range(world)]
        h0s = [torch.zeros_like(h0) for _ in range(world)]
        dist.all_gather(hs, m.h)
        dist.all_gather(h0s, h0)
        if rank == 0:
            # single-GPU reference: all 256 experts on one device, same weights
            full = []
            for l in range(2):
                parts = [synth.make_experts(m.epr, 2048, 512, seed=0 + 1000 * l + r, device=dev,
                                            chunk=16) for r in range(world)]
                full.append(synth.HostExperts(256, *(torch.cat([getattr(p, n) for p in parts])
                                                     for n in ("w13_weight", "w2_weight",
                                                               "w13_scale_inv", "w2_scale_inv"))))
            h = torch.cat(h0s)
            for l in range(2):
                ids, w = moe.router_topk(h, m.gate[l], 8)
                ids = torch.from_numpy(tr[0, l].astype("int32")).to(dev)
                moe.fp8_moe_forward(h, ids, w, full[l].w13_weight, full[l].w13_scale_inv,
                                    full[l].w2_weight, full[l].w2_scale_inv, out=h, accumulate=True)
            got = torch.cat(hs).float()
            err = float((got - h.float()).abs().max() / h.float().abs().max())
            q.put((rank, err))
        else:
            q.put((rank, 0.0))
        dist.barrier()
    except Exception as exc:
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not cuda_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_ep_two_gpus_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert isinstance(res[0], float) and res[0] < 1e-2, res
    assert res[1] == 0.0, res
