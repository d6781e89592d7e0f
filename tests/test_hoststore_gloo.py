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


def _node_worker(rank, world, port, q, nodes, node_free):
    """Ranks whose GPUs sit on ``nodes`` (faked), each node reporting
    ``node_free`` free bytes."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from drama3_offloading_b200 import hoststore
        hoststore.node_mem_free = lambda n: node_free
        st = hoststore.SharedHostStore(1 << 20, local_rank=rank, group=dist.group.WORLD,
                                       headroom=0, node=nodes[rank])
        a = st.take((256,), torch.int64)
        if st.primary:
            a.copy_(torch.arange(256) * 7)
        dist.barrier()
        if st.copies > 1:
            st.copy_from_primary()
            dist.barrier()
        same = bool((a == torch.arange(256) * 7).all())
        dist.barrier()
        # the last rank writes its copy; who sees it tells which ranks share it
        if rank == world - 1:
            a[0] = -1
        dist.barrier()
        q.put((rank, (st.copies, st.owner, same, int(a[0]) == -1)))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def _run_nodes(nodes, node_free):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = len(nodes)
    procs = [ctx.Process(target=_node_worker, args=(r, world, port, q, nodes, node_free))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return res


def test_one_copy_per_numa_node():
    # GPUs on nodes 0, 1, 1: two copies with the same bytes; rank 2 shares
    # rank 1's copy (its write is seen by rank 1, not by rank 0)
    res = _run_nodes([0, 1, 1], 1 << 40)
    assert res == {0: (2, True, True, False), 1: (2, True, True, True),
                   2: (2, False, True, True)}, res


def test_one_copy_when_nodes_unknown_or_short_of_ram():
    # a node that cannot hold a copy, or a GPU whose node is unknown: one copy
    for nodes, free in (([0, 1], 1 << 20), ([-1, 0], 1 << 40)):
        res = _run_nodes(nodes, free)
        assert res == {0: (1, True, True, True), 1: (1, False, True, True)}, (nodes, res)


def test_single_rank_store_places_on_its_node():
    from drama3_offloading_b200.hoststore import SharedHostStore
    st = SharedHostStore(1 << 20, headroom=0, node=0)
    a = st.take((4096,), torch.uint8)
    a.fill_(3)
    assert st.copies == 1 and st.owner and st.primary and st.node == 0
    assert isinstance(st.bound, bool) and int(a.sum()) == 3 * 4096
