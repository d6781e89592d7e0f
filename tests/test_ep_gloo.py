"""Expert-parallel exchange on CPU (gloo, world size 2).

Each rank routes its tokens to experts sharded over both ranks, packs them
into the static-capacity layout (tests/ep_reference.py restates
d3_ep_dispatch_pack), exchanges with ``ep.exchange`` (all-to-all with equal
splits), applies a per-expert function on the receiving rank, exchanges back
and combines; the result must equal a single-process computation.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        import ep_reference as ref
        from drama3_offloading_b200 import ep
        E, T, k, H = 8, 5, 3, 16
        epr, cap = E // world, T * k
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(T, H, generator=g)
        ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k, generator=g)
        send_x, send_eid, src = ref.pack(x, ids, world, epr, cap)
        recv_x = torch.empty_like(send_x)
        recv_eid = torch.empty_like(send_eid)
        ep.exchange(send_x, recv_x)
        ep.exchange(send_eid, recv_eid)
        # local "expert": global expert id g multiplies its row by (g + 1)
        gid = recv_eid.to(torch.float32) + rank * epr
        y = torch.where(recv_eid[:, None] >= 0, recv_x * (gid[:, None] + 1), torch.zeros_like(recv_x))
        ret = torch.empty_like(y)
        ep.exchange(y, ret)
        got = ref.combine(ret, src, w)
        want = torch.zeros(T, H)
        for t in range(T):
            for j in range(k):
                want[t] += w[t, j] * x[t] * (int(ids[t, j]) + 1)
        q.put((rank, bool(torch.allclose(got, want, atol=1e-5, rtol=1e-5))))
    except Exception as exc:
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res
