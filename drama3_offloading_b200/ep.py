"""Fully HBM-resident expert-parallel MoE decode.

256 experts per layer are sharded evenly over the N ranks (32 per GPU at
N = 8) and stay resident in HBM; the global decode batch (64 streams) is
split over the ranks (64/N tokens each).  Per layer and step, on every rank:

    router (local tokens) -> d3_ep_dispatch_p2p: token rows and local expert
    ids stored straight into the destination ranks' exchange buffers over
    NVLink (static capacity per peer), epoch flag released on each
    -> d3_ep_wait (all sources arrived) -> d3_moe_fp8_forward over the
    received rows (one expert per row) -> d3_ep_return_p2p: outputs stored
    back into the source ranks' buffers -> d3_ep_wait
    -> d3_ep_combine: h += sum_k w[t,k] y[t,k]

``exchange="nccl"`` runs the same step with NCCL all-to-alls instead (pack
locally, all-to-all rows and ids, all-to-all outputs back).

Every buffer has a fixed shape (capacity = local pairs per peer), so the step
needs no host sync and is captured into one CUDA graph, collectives included.
At N = 1 the exchange disappears and the layer is one fp8_moe_forward.

Errors: every NVLink wait is bounded (2 s of GPU time).  A wait that runs out
records a code in the device error word and the step goes on -- it cannot
stop mid-graph -- so that step's hidden states are wrong.  The step itself
never reads the word (that would sync the host every step): call
``check()`` (or ``moe.check_errors()``) after ``step()`` or after replaying
the captured graph, or pass ``step(check=True)``; ``close()`` checks once
more and raises after tearing the exchange down.

No counterpart in the reference (it has no multi-GPU code).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib, moe, synth


def exchange(send: torch.Tensor, recv: torch.Tensor, group=None) -> None:
    """Static all-to-all: row block r of ``send`` goes to rank r, the block
    from rank r lands in row block r of ``recv`` (equal splits)."""
    import torch.distributed as dist
    dist.all_to_all_single(recv, send, group=group)


def _al(v: int) -> int:
    return (v + 255) // 256 * 256


class P2PExchange:
    """Every rank's exchange buffer (recv_x, recv_eid, ret, flag_d, flag_r;
    layout of csrc/ep_p2p.cu) in its own HBM, mapped into every rank's
    process through CUDA IPC, and the per-peer device pointers the kernels
    store into.  The handles travel once over the process group at setup."""

    def __init__(self, rank: int, world: int, cap: int, H: int, device, group=None):
        import torch.distributed as dist
        if world > 16:
            raise ValueError("the NVLink exchange takes at most 16 ranks")
        self.rank, self.world = rank, world
        n = world * cap
        self.off = {}
        o = 0
        for name, nbytes in (("recv_x", n * H * 2), ("recv_eid", n * 4), ("ret", n * H * 2),
                             ("flag_d", world * 8), ("flag_r", world * 8)):
            self.off[name] = o
            o += _al(nbytes)
        self.buf = torch.zeros(o, dtype=torch.uint8, device=device)
        view = lambda name, nbytes, dt: self.buf[self.off[name]:self.off[name] + nbytes].view(dt)
        self.recv_x = view("recv_x", n * H * 2, torch.bfloat16).view(n, H)
        self.recv_eid = view("recv_eid", n * 4, torch.int32)
        self.ret = view("ret", n * H * 2, torch.bfloat16).view(n, H)
        self.flag_d = view("flag_d", world * 8, torch.int64)
        self.flag_r = view("flag_r", world * 8, torch.int64)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.counters = torch.zeros(2, dtype=torch.int32, device=device)
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_uint64()
        _lib.call("d3_ipc_get", _lib.ptr(self.buf), handle, ctypes.byref(offset))
        infos = [None] * world
        dist.all_gather_object(infos, (bytes(handle), offset.value), group=group)
        self.opened = []
        bases = []
        for r, (h, off) in enumerate(infos):
            if r == rank:
                bases.append(self.buf.data_ptr())
                continue
            b = ctypes.c_void_p()
            _lib.call("d3_ipc_open", ctypes.create_string_buffer(h, 64), ctypes.byref(b))
            self.opened.append(b.value)
            bases.append(b.value + off)
        arr = lambda name: (ctypes.c_void_p * world)(*(b + self.off[name] for b in bases))
        self.peer = {name: arr(name) for name in self.off}
        dist.barrier(group=group)

    def close(self) -> None:
        for b in self.opened:
            _lib.call("d3_ipc_close", ctypes.c_void_p(b))
        self.opened = []


class ExpertParallelMoE:
    def __init__(self, layers: int = 40, experts: int = 256, hidden: int = 2048,
                 inter: int = 512, topk: int = 8, global_batch: int = 64, rank: int = 0,
                 world: int = 1, group=None, device="cuda", seed: int = 0,
                 trace: np.ndarray | None = None, exchange: str = "p2p"):
        if experts % world or global_batch % world:
            raise ValueError("experts and global_batch must divide evenly over the ranks")
        self.device = dev = torch.device(device)
        self.L, self.E, self.H, self.I, self.k = layers, experts, hidden, inter, topk
        self.rank, self.world, self.group = rank, world, group
        self.epr = experts // world
        self.T = global_batch // world
        self.cap = self.T * topk                    # pairs this rank can send to one peer
        g = torch.Generator(device=dev).manual_seed(seed + 11)
        # resident local experts: layer l, global experts [rank*epr, (rank+1)*epr)
        self.w = [synth.make_experts(self.epr, hidden, inter, seed=seed + 1000 * l + rank,
                                     device=dev, chunk=16) for l in range(layers)]
        self.gate = [(torch.randn(experts, hidden, generator=g, device=dev) * 0.02)
                     .to(torch.bfloat16) for _ in range(layers)]
        self.h = torch.randn(self.T, hidden, generator=g, device=dev).to(torch.bfloat16)
        self.ids = torch.empty(self.T, topk, dtype=torch.int32, device=dev)
        self.wts = torch.empty(self.T, topk, dtype=torch.float32, device=dev)
        n = world * self.cap
        self.send_x = torch.zeros(n, hidden, dtype=torch.bfloat16, device=dev)
        self.recv_x = torch.zeros_like(self.send_x)
        self.send_eid = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.recv_eid = torch.full_like(self.send_eid, -1)
        self.y = torch.zeros_like(self.send_x)
        self.ret = torch.zeros_like(self.send_x)
        self.src_slot = torch.full((self.T, topk), -1, dtype=torch.int32, device=dev)
        self.ones = torch.ones(n, 1, dtype=torch.float32, device=dev)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=dev)
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.exchange = exchange if world > 1 else "none"
        self.p2p = P2PExchange(rank, world, self.cap, hidden, dev, group) \
            if self.exchange == "p2p" else None
        if trace is None:
            from .trace import uniform_trace
            trace = uniform_trace(steps=256, tokens=global_batch, layers=layers,
                                  experts=experts, k=topk)
        # this rank's tokens of each step: [steps, layers, T, k]
        mine = trace[:, :, rank * self.T:(rank + 1) * self.T, :]
        self.trace_steps = mine.shape[0]
        self.trace_dev = torch.from_numpy(np.ascontiguousarray(mine).astype(np.int32)).to(dev)
        self.step_idx = torch.zeros(1, dtype=torch.int64, device=dev)
        self.graph = None
        moe.router_topk(self.h, self.gate[0], topk, out_ids=self.ids, out_w=self.wts)

    # ------------------------------------------------------------ one step
    def _layer(self, l: int, ids: torch.Tensor, gemm_events: list | None = None,
               xchg_events: list | None = None) -> None:
        h = self.h
        moe.router_topk(h, self.gate[l], self.k, out_ids=self.ids, out_w=self.wts)
        w = self.w[l]
        if self.world == 1:
            if gemm_events is not None:
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
            moe.fp8_moe_forward(h, ids, self.wts, w.w13_weight, w.w13_scale_inv, w.w2_weight,
                                w.w2_scale_inv, out=h, accumulate=True)
            if gemm_events is not None:
                e1.record()
                gemm_events.append((e0, e1))
            return
        st = _lib.stream_ptr()
        if self.p2p is not None:
            self._layer_p2p(l, ids, w, st, gemm_events, xchg_events)
            return
        _lib.call("d3_ep_dispatch_pack", _lib.ptr(h), _lib.ptr(ids), self.T, self.k, self.H,
                  self.world, self.epr, self.cap, _lib.ptr(self.send_x), _lib.ptr(self.send_eid),
                  _lib.ptr(self.src_slot), _lib.ptr(self.overflow), st)
        exchange(self.send_x, self.recv_x, self.group)
        exchange(self.send_eid, self.recv_eid, self.group)
        if gemm_events is not None:
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
        moe.fp8_moe_forward(self.recv_x, self.recv_eid.view(-1, 1), self.ones, w.w13_weight,
                            w.w13_scale_inv, w.w2_weight, w.w2_scale_inv, out=self.y)
        if gemm_events is not None:
            e1.record()
            gemm_events.append((e0, e1))
        exchange(self.y, self.ret, self.group)
        _lib.call("d3_ep_combine", _lib.ptr(self.ret), _lib.ptr(self.src_slot),
                  _lib.ptr(self.wts), 1, self.T, self.k, self.H, _lib.ptr(h), 1, st)

    WAIT_BUDGET_NS = 2_000_000_000

    def _layer_p2p(self, l, ids, w, st, gemm_events, xchg_events=None) -> None:
        """The same layer with the exchange over NVLink peer stores, in three C
        calls: the dispatch stores the rows into the peers; the expert call
        waits for every source's rows (in its route launch) and stores each
        served row back into its source (in its combine launch); the combine
        waits for every serving rank's rows.  ``xchg_events`` receives CUDA
        event pairs around the dispatch and around the combine (its wait for
        the slowest serving rank included)."""
        x = self.p2p
        err = moe.error_word(self.device)
        if xchg_events is not None:
            d0, d1 = torch.cuda.Event(True), torch.cuda.Event(True)
            d0.record()
        _lib.call("d3_ep_dispatch_p2p", _lib.ptr(self.h), _lib.ptr(ids), self.T, self.k, self.H,
                  self.world, self.rank, self.epr, self.cap, x.peer["recv_x"],
                  x.peer["recv_eid"], x.peer["flag_d"], _lib.ptr(self.src_slot),
                  _lib.ptr(self.overflow), _lib.ptr(x.epoch), _lib.ptr(x.counters), st)
        if xchg_events is not None:
            d1.record()
        if gemm_events is not None:
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
        moe.fp8_moe_forward_p2p(x.recv_x, x.recv_eid.view(-1, 1), self.ones, w.w13_weight,
                                w.w13_scale_inv, w.w2_weight, w.w2_scale_inv,
                                wait_flags=x.flag_d, epoch=x.epoch, n_ranks=self.world,
                                rank=self.rank, cap=self.cap, peer_ret=x.peer["ret"],
                                peer_flag_r=x.peer["flag_r"], counter=x.counters[1:],
                                wait_code=31, budget_ns=self.WAIT_BUDGET_NS)
        if gemm_events is not None:
            e1.record()
            gemm_events.append((e0, e1))
        if xchg_events is not None:
            c0, c1 = torch.cuda.Event(True), torch.cuda.Event(True)
            c0.record()
        _lib.call("d3_ep_combine_p2p", _lib.ptr(x.ret), _lib.ptr(self.src_slot),
                  _lib.ptr(self.wts), 1, self.T, self.k, self.H, _lib.ptr(self.h), 1,
                  _lib.ptr(x.flag_r), self.world, _lib.ptr(x.epoch), _lib.ptr(err), 32,
                  self.WAIT_BUDGET_NS, st)
        if xchg_events is not None:
            c1.record()
            xchg_events.append((d0, d1, c0, c1))

    def check(self) -> None:
        """Raise if a bounded NVLink wait of an earlier step ran out (reads the
        device error word: synchronises the host with the device)."""
        moe.check_errors(self.device)

    def close(self) -> None:
        """Unmap the peers' exchange buffers (after the last step, on every
        rank), then raise if any step's bounded wait ran out."""
        torch.cuda.synchronize(self.device)
        code = int(moe.error_word(self.device).item())
        self.graph = None
        if self.p2p is not None:
            import torch.distributed as dist
            dist.barrier(group=self.group)
            self.p2p.close()
            self.p2p = None
        if code:
            raise RuntimeError(f"d3 device error code {code}: {moe.error_message(code)} "
                               "(a bounded wait expired during an earlier step)")

    def step(self, gemm_events: list | None = None, check: bool = False,
             xchg_events: list | None = None) -> None:
        """One decode step of all layers (eager; capturable).  ``check=True``
        synchronises afterwards and raises if a bounded wait ran out (not
        inside a capture).  The event lists (eager timing only) receive CUDA
        event pairs around each layer's expert call, and around its NVLink
        dispatch and combine."""
        cur = self.trace_dev.index_select(0, self.step_idx)[0]
        self.step_idx.add_(1).remainder_(self.trace_steps)
        for l in range(self.L):
            self._layer(l, cur[l], gemm_events, xchg_events)
        if check:
            self.check()

    def capture(self) -> torch.cuda.CUDAGraph:
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.step()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.graph = g
        return g

    def local_expert_bytes(self) -> int:
        return synth_expert_bytes(self.H, self.I)


def synth_expert_bytes(H: int, I: int) -> int:
    return 3 * H * I + 3 * H * I * 4 // (128 * 128)
