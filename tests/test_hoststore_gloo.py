"""Multi-rank host logic on CPU (gloo, world size 2): the shared expert store
that every local rank of a multi-GPU run maps (one copy of the 30 GiB of
experts per machine instead of one per rank), and the RAM guard that refuses
a store the machine cannot hold.  No GPU: page-locking is skipped here."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
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
        from drama3_offloading_b200.hoststore import SharedHostStore
        st = SharedHostStore(1 << 20, local_rank=rank, group=dist.group.WORLD, headroom=0)
        a = st.take((256,), torch.int64)
        b = st.take((3, 5), torch.float32)
        if rank == 0:
            a.copy_(torch.arange(256) * 7)
            b.fill_(2.5)
        dist.barrier()
        ok = bool((a == torch.arange(256) * 7).all()) and bool((b == 2.5).all())
        # page alignment of the sub-tensors
        ok = ok and (b.data_ptr() - a.data_ptr()) % 4096 == 0
        # a write by rank 1 is seen by rank 0 (one physical copy)
        if rank == 1:
            a[0] = -1
        dist.barrier()
        ok = ok and int(a[0]) == -1
        q.put((rank, ok))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_shared_store_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res


def _oom_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from drama3_offloading_b200.hoststore import SharedHostStore
        try:
            SharedHostStore(1 << 60, local_rank=rank, group=dist.group.WORLD)
            q.put((rank, "allocated"))
        except MemoryError as exc:
            q.put((rank, "refused" if "available" in str(exc) else repr(exc)))
    finally:
        dist.destroy_process_group()


def test_store_larger_than_ram_is_refused_on_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_oom_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "refused", 1: "refused"}, res
