"""CPU ORACLE -- test infrastructure only.

Restates the reference's hot-path semantics on the CPU so that tests/,
``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` / ``--impl reference``
leg can CHECK (or time, as the CPU baseline) the CUDA path.  The product path
never imports this package; the package ``drama3_offloading_b200`` fails loudly
when its CUDA library is missing instead of falling back to anything here.

Contents and what each follows:

* ``resolve`` / ``resolve_lfu`` / ``fetch`` / ``replay`` -- the C restatement in
  ``oracle/resolve.c`` of ``_resolve_slots`` (bin/devcache.py:45-98) and
  ``_fetch_experts`` (bin/devcache.py:101-130; csrc/fetch_experts.cu:49-69).
  PINNED: checked bit for bit against the reference's own Triton kernels run
  under ``TRITON_INTERPRET=1`` (fixtures in tests/golden/, made by
  tests/golden/make_golden.py).
* ``router_topk`` -- the upstream fish-speech MoE router (gate Linear, softmax,
  top-k, ``norm_topk_prob`` renormalisation), quoted in the reference at
  notes/01-static-findings.md:133-138.  Logits are defined as the exactly
  rounded bf16 of the dot product (fp64 accumulation, then fp32, then bf16,
  both round-to-nearest-even); top-k ties go to the lower expert index.
* ``dequantize_fp8_blocks`` / ``moe_forward`` -- the upstream dequantise-then-
  matmul MoE path (``expert_weights``/``dequantize_fp8_blocks``/
  ``forward_gathered``, quoted at notes/13-non-ada-gpus.md:37-54) with SwiGLU
  experts (``hidden_act: silu``, notes/drama3-config.json:91) and the weighted
  top-k sum.  The upstream module (fish-speech @ 5415669) is not vendored in
  the reference, so the absolute MoE numerics are PARITY UNPINNED: only the
  cache/fetch/slot semantics above are pinned to the reference's own code.
* ``shared_expert_forward`` -- Drama-3's per-layer bf16 shared expert with its
  sigmoid gate (inferred from the config, see the function), fp32.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

_HERE = Path(__file__).resolve().parent
_LIB = None

__all__ = [
    "lib", "init_tables", "resolve", "resolve_lfu", "fetch", "replay",
    "bf16_round", "router_logits", "router_topk", "dequantize_fp8_blocks",
    "quantize_fp8_blocks", "moe_forward", "shared_expert_forward",
]


def lib() -> ctypes.CDLL:
    """Load (building if needed) oracle/liboracle.so."""
    global _LIB
    if _LIB is not None:
        return _LIB
    so = _HERE / "liboracle.so"
    src = _HERE / "resolve.c"
    if not so.exists() or so.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    L = ctypes.CDLL(str(so))
    P = ctypes.c_void_p
    i32, i64 = ctypes.c_int32, ctypes.c_int64
    L.oracle_init.argtypes = [P, ctypes.c_int, P, P, ctypes.c_int, P]
    L.oracle_resolve.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P, P, ctypes.c_int,
                                 P, P, P, P, P]
    L.oracle_resolve.restype = ctypes.c_int
    L.oracle_resolve_lfu.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P, P, P, P,
                                     ctypes.c_int, P, P, P, P, P]
    L.oracle_resolve_lfu.restype = ctypes.c_int
    L.oracle_fetch.argtypes = [P, P, P, P, ctypes.c_int, i64]
    L.oracle_replay.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, P, P, P, P]
    L.oracle_replay.restype = ctypes.c_int
    del i32
    _LIB = L
    return L


def _p(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


class Tables:
    """Host copy of one layer's cache tables (bin/devcache.py:146-152)."""

    def __init__(self, num_experts: int, capacity: int):
        self.E, self.C = num_experts, capacity
        self.slot_of = np.empty(num_experts, np.int32)
        self.slot_expert = np.empty(capacity, np.int32)
        self.stamp = np.empty(capacity, np.int64)
        self.step = np.zeros(1, np.int64)
        self.freq = np.zeros(capacity, np.int64)
        self.ins = -np.arange(capacity, 0, -1, dtype=np.int64)
        lib().oracle_init(_p(self.slot_of), num_experts, _p(self.slot_expert), _p(self.stamp),
                          capacity, _p(self.step))


def init_tables(num_experts: int, capacity: int) -> Tables:
    return Tables(num_experts, capacity)


def resolve(t: Tables, ids) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """One ``_resolve_slots`` call. Returns (out_slot[k], fetch_slot[nmiss],
    fetch_expert[nmiss], nmiss) and updates ``t`` in place."""
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
    k = ids.size
    out = np.zeros(k, np.int32)
    fs = np.zeros(k, np.int32)
    fe = np.zeros(k, np.int32)
    nm = np.zeros(1, np.int32)
    lib().oracle_resolve(_p(ids), k, _p(t.slot_of), t.E, _p(t.slot_expert), _p(t.stamp), t.C,
                         _p(out), _p(fs), _p(fe), _p(nm), _p(t.step))
    n = int(nm[0])
    return out, fs[:n].copy(), fe[:n].copy(), n


def resolve_lfu(t: Tables, ids) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
    k = ids.size
    out = np.zeros(k, np.int32)
    fs = np.zeros(k, np.int32)
    fe = np.zeros(k, np.int32)
    nm = np.zeros(1, np.int32)
    lib().oracle_resolve_lfu(_p(ids), k, _p(t.slot_of), t.E, _p(t.slot_expert), _p(t.stamp),
                             _p(t.freq), _p(t.ins), t.C, _p(out), _p(fs), _p(fe), _p(nm),
                             _p(t.step))
    n = int(nm[0])
    return out, fs[:n].copy(), fe[:n].copy(), n


def fetch(src: np.ndarray, dst: np.ndarray, idx, slot, njobs: int, expert_bytes: int) -> None:
    idx = np.ascontiguousarray(np.asarray(idx, np.int32))
    slot = np.ascontiguousarray(np.asarray(slot, np.int32))
    lib().oracle_fetch(_p(src), _p(dst), _p(idx), _p(slot), int(njobs), int(expert_bytes))


def replay(trace: np.ndarray, num_experts: int, capacity: int, policy: str = "lru",
           want_slots: bool = False):
    """Replay an ``int16 [steps, layers, k]`` trace; returns dict with hits,
    misses, misses_per_step and optionally out_slots."""
    trace = np.ascontiguousarray(trace, dtype=np.int16)
    steps, layers, k = trace.shape
    if k > 64:
        raise ValueError("k <= 64")
    mps = np.zeros(steps, np.int32)
    h = np.zeros(1, np.int64)
    m = np.zeros(1, np.int64)
    slots = np.zeros((steps, layers, k), np.int32) if want_slots else None
    rc = lib().oracle_replay(_p(trace), steps, layers, k, num_experts, capacity,
                             1 if policy == "lfu" else 0, _p(mps), _p(h), _p(m),
                             _p(slots) if want_slots else None)
    if rc != 0:
        raise MemoryError("oracle_replay")
    return {"hits": int(h[0]), "misses": int(m[0]), "misses_per_step": mps, "out_slots": slots}


# ---------------------------------------------------------------- numerics

def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 round-to-nearest-even, returned as float32 values."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    out = np.where(nan, np.float32(np.nan), out)
    return out


def router_logits(x: torch.Tensor, gate_w: torch.Tensor) -> torch.Tensor:
    """Exactly rounded bf16 router logits ``x @ gate_w.T`` -> float32 [T, E]."""
    xd = x.to(torch.float64).numpy()
    wd = gate_w.to(torch.float64).numpy()
    acc = xd @ wd.T
    return torch.from_numpy(bf16_round(acc.astype(np.float32)))


def router_topk(x: torch.Tensor, gate_w: torch.Tensor, k: int = 8, renorm: bool = True):
    """Upstream MoE router. Returns (ids int32 [T,k], weights float32 [T,k],
    logits float32 [T,E], ties int = number of rows whose k-th and (k+1)-th
    logits are equal)."""
    logits = router_logits(x, gate_w)
    T, E = logits.shape
    lg = logits.numpy()
    # stable descending sort on the logit, ties -> lower index first
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -lg), axis=-1)[:, :k]
    ids = order.astype(np.int32)
    top = np.take_along_axis(lg, order, axis=-1).astype(np.float64)
    mx = lg.max(axis=-1, keepdims=True).astype(np.float64)
    ex_all = np.exp(lg.astype(np.float64) - mx)
    p = np.exp(top - mx) / ex_all.sum(axis=-1, keepdims=True)
    if renorm:
        p = p / p.sum(axis=-1, keepdims=True)
    srt = -np.sort(-lg, axis=-1)
    ties = int((srt[:, k - 1] == srt[:, k]).sum()) if k < E else 0
    return torch.from_numpy(ids), torch.from_numpy(p.astype(np.float32)), logits, ties


def quantize_fp8_blocks(w: torch.Tensor, block: int = 128):
    """fp32 [..., R, C] -> (e4m3 [..., R, C], fp32 scale_inv [..., R/128, C/128])
    with ``scale_inv = amax/448`` per 128x128 block and ``q = e4m3(w/scale_inv)``."""
    *lead, R, C = w.shape
    rb, cb = (R + block - 1) // block, (C + block - 1) // block
    wp = torch.nn.functional.pad(w, (0, cb * block - C, 0, rb * block - R))
    blk = wp.reshape(*lead, rb, block, cb, block)
    amax = blk.abs().amax(dim=(-3, -1))
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (blk / s[..., :, None, :, None]).reshape(*lead, rb * block, cb * block)[..., :R, :C]
    return q.to(torch.float8_e4m3fn), s.to(torch.float32)


def dequantize_fp8_blocks(w: torch.Tensor, scale_inv: torch.Tensor,
                          dtype=torch.float32, block: int = 128) -> torch.Tensor:
    """``w.float() * scale_inv`` broadcast over 128x128 blocks, cast to dtype."""
    R, C = w.shape[-2], w.shape[-1]
    s = scale_inv.to(torch.float32).repeat_interleave(block, -2).repeat_interleave(block, -1)
    return (w.to(torch.float32) * s[..., :R, :C]).to(dtype)


def moe_forward(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, w13: torch.Tensor,
                s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
                dtype=torch.float32) -> torch.Tensor:
    """Dequantise-then-matmul routed MoE on the CPU.

    x [T,H]; ids [T,k] index dim 0 of w13/w2; weights [T,k]; w13 [n,2I,H] e4m3
    (gate rows [0,I), up rows [I,2I)); s13 [n,2I/128,H/128]; w2 [n,H,I] e4m3;
    s2 [n,H/128,I/128].  For each (t,k): h = silu(x W_g^T) * (x W_u^T),
    out_t += w_tk * h W_d^T.  Accumulates in ``dtype`` (float32 or float64);
    with bfloat16 it rounds like the upstream bf16 path.  Returns float32 [T,H].
    """
    T, H = x.shape
    I = w13.shape[1] // 2
    xs = x.to(dtype)
    out = torch.zeros(T, H, dtype=torch.float64 if dtype == torch.float64 else torch.float32)
    flat = ids.reshape(-1).to(torch.int64)
    for e in torch.unique(flat).tolist():
        rows = (ids.to(torch.int64) == e).nonzero()
        t_idx, k_idx = rows[:, 0], rows[:, 1]
        W13 = dequantize_fp8_blocks(w13[e], s13[e], dtype)
        W2 = dequantize_fp8_blocks(w2[e], s2[e], dtype)
        xe = xs[t_idx]
        gu = xe @ W13.T
        g, u = gu[:, :I], gu[:, I:]
        h = torch.nn.functional.silu(g) * u
        y = (h @ W2.T).to(out.dtype)
        wk = weights[t_idx, k_idx].to(out.dtype)[:, None]
        out.index_add_(0, t_idx, y * wk)
    return out.to(torch.float32)

def shared_expert_forward(x: torch.Tensor, w13_s: torch.Tensor, w2_s: torch.Tensor,
                          gate_s: torch.Tensor | None) -> torch.Tensor:
    """Drama-3's shared expert on the CPU, fp32: bf16 w13_s [2I, H] (gate rows
    [0, I), up rows [I, 2I)), w2_s [H, I]; out = sigmoid(x . gate_s) *
    (silu(x W_g^T) * (x W_u^T)) W_d^T, ungated when gate_s is None.  The
    upstream block runs it beside the routed experts for every token
    (notes/01-static-findings.md:80-82; ``shared_expert_gate: true`` and
    ``shared_expert_intermediate_size: 512``, notes/drama3-config.json:215-216;
    the sigmoid gate follows the usual shared-expert gating and is inferred).
    Returns float32 [T, H]."""
    I = w13_s.shape[0] // 2
    xf = x.float()
    gu = xf @ w13_s.float().T
    h = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    y = h @ w2_s.float().T
    if gate_s is not None:
        y = y * torch.sigmoid(xf @ gate_s.float().reshape(-1))[:, None]
    return y
