"""Router and FP8 expert computation -- the calls the reference makes into
upstream fish-speech, served by libd3b200.so.

* ``router_topk(x, gate_w, k, renorm)`` -- the MoE block's gate -> softmax ->
  top-k -> renorm (fish-speech moe.py:217-220, quoted in the reference at
  notes/01-static-findings.md:133-138).
* ``fp8_moe_forward(x, ids, w, w13, s13, w2, s2)`` -- same signature and
  meaning as upstream ``fp8_moe_forward`` as the reference calls it
  (bin/devcache.py:275-277, bin/offload.py:177, :239, :340, :388, :449):
  ``ids`` index dim 0 of the weight stacks (expert ids, cache slots or a
  renumbered subset), ``w`` are the routing weights, the result is bf16.

Workspaces are allocated once per (device, size) and reused, so repeated
calls -- and CUDA-graph capture -- do not allocate.  Kernel-side failures
(a bounded wait that timed out) set a device error word instead of hanging;
``check_errors()`` reads it (synchronising).
"""
from __future__ import annotations

import torch

from . import _lib

_WS: dict = {}
_ERR: dict = {}


def _workspace(device: torch.device, nbytes: int, tag: str, zero: bool = False) -> torch.Tensor:
    key = (tag, device.index)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def error_word(device: torch.device) -> torch.Tensor:
    t = _ERR.get(device.index)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[device.index] = t
    return t


# device error codes: which bounded wait gave up
ERROR_CODES = {
    1: "expert GEMM: the TMA producer waited for a free pipeline stage",
    2: "expert GEMM: the MMA issuer waited for loaded operands or a free accumulator",
    3: "expert GEMM: the final wait for the CTA's own MMAs",
    4: "expert GEMM: the epilogue waited for an accumulator",
    5: "expert call (one launch): a grid-wide phase barrier or the down-projection operand gate",
    31: "expert parallel: a source rank's dispatch never arrived",
    32: "expert parallel: a serving rank's returned rows never arrived",
    41: "decode overlap: a fetched expert's bytes never landed",
}


def error_message(code: int) -> str:
    return ERROR_CODES.get(code, "unknown bounded wait")


def check_errors(device=None) -> None:
    """Raise if a kernel on ``device`` gave up on a bounded wait (the error
    word keeps the first code; see ERROR_CODES)."""
    device = torch.device(device or torch.cuda.current_device())
    if device.type != "cuda":
        device = torch.device("cuda", torch.cuda.current_device())
    v = int(error_word(device).item())
    if v:
        raise RuntimeError(f"d3 device error code {v}: {error_message(v)} (a bounded wait "
                           "expired)")


def router_topk(x: torch.Tensor, gate_w: torch.Tensor, k: int = 8, renorm: bool = True,
                out_ids: torch.Tensor | None = None, out_w: torch.Tensor | None = None,
                out_w_bf16: torch.Tensor | None = None, stream=None):
    """x bf16 [T,H], gate_w bf16 [E,H] -> (ids int32 [T,k], weights f32 [T,k])."""
    if x.dtype != torch.bfloat16 or gate_w.dtype != torch.bfloat16:
        raise TypeError("router_topk expects bf16 x and gate_w")
    x = x.contiguous()
    gate_w = gate_w.contiguous()
    T, H = x.shape
    E = gate_w.shape[0]
    dev = x.device
    ids = out_ids if out_ids is not None else torch.empty(T, k, dtype=torch.int32, device=dev)
    w = out_w if out_w is not None else torch.empty(T, k, dtype=torch.float32, device=dev)
    need = _lib.load().d3_router_workspace_size(T, E)
    ws = _workspace(dev, need, "router")
    _lib.call("d3_router_topk", _lib.ptr(x), _lib.ptr(gate_w), T, H, E, k, 1 if renorm else 0,
              _lib.ptr(ids), _lib.ptr(w), _lib.ptr(out_w_bf16), _lib.ptr(ws), ws.numel(),
              _lib.stream_ptr(stream))
    return ids, w


def workspace_bytes(T: int, topk: int, n_experts: int, H: int, I: int) -> int:
    return int(_lib.load().d3_moe_workspace_size(T, topk, n_experts, H, I))


SHARED_FUSED_MAX_PAIRS = 32   # the decode (GEMV) path of the library


def fp8_moe_forward(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                    w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
                    out: torch.Tensor | None = None, accumulate: bool = False,
                    stream=None, shared: tuple | None = None) -> torch.Tensor:
    """Routed MoE over block-scaled FP8 experts; returns bf16 [T, H].

    ids (int32/int64) out of range -- e.g. -1 -- contribute nothing.  With
    ``accumulate=True`` the result is added to ``out`` (which may be ``x``
    itself: the block's residual add).

    ``shared=(w13_s, w2_s, gate_s)`` adds Drama-3's shared expert: bf16
    w13_s [2I, H] (gate rows, then up rows), w2_s [H, I], gate_s [H] or None,
    ``sigmoid(x . gate_s) * w2_s(silu(x w_g^T) * (x w_u^T))``.  Decode batches
    run it inside the same two launches as the routed experts
    (``d3_moe_fp8_forward_shared``); larger batches add it with two plain
    bf16 GEMMs (cuBLAS) after the routed call."""
    if x.dtype != torch.bfloat16:
        raise TypeError("x must be bf16")
    x = x.contiguous()
    T, H = x.shape
    ids = ids.reshape(T, -1)
    topk = ids.shape[1]
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    weights = weights.reshape(T, topk)
    if weights.dtype not in (torch.float32, torch.bfloat16):
        weights = weights.to(torch.float32)
    weights = weights.contiguous()
    n, two_i, h2 = w13.shape
    if h2 != H or w2.shape[0] != n or w2.shape[1] != H:
        raise ValueError("weight shapes do not match x")
    I = two_i // 2
    for t, name in ((w13, "w13"), (w2, "w2")):
        if t.element_size() != 1 or not t.is_contiguous():
            raise TypeError(f"{name} must be a contiguous 1-byte (e4m3) tensor")
    s13 = s13.contiguous()
    s2 = s2.contiguous()
    if s13.dtype != torch.float32 or s2.dtype != torch.float32:
        raise TypeError("scales must be float32")
    dev = x.device
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs an out tensor")
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or not out.is_contiguous() or tuple(out.shape) != (T, H):
        raise ValueError("out must be a contiguous bf16 [T, H] tensor")
    need = workspace_bytes(T, topk, n, H, I)
    if need == 0:
        raise ValueError(f"unsupported MoE shape T={T} topk={topk} n={n} H={H} I={I}")
    ws = _workspace(dev, need, "moe")
    wf = 1 if weights.dtype == torch.float32 else 0
    if shared is not None:
        sw13, sw2, sg = shared
        for t, name in ((sw13, "w13_s"), (sw2, "w2_s")):
            if t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise TypeError(f"shared expert {name} must be contiguous bf16")
        if tuple(sw13.shape) != (2 * I, H) or tuple(sw2.shape) != (H, I):
            raise ValueError("shared expert shapes must be w13_s [2I, H] and w2_s [H, I]")
        if sg is not None:
            sg = sg.reshape(H).contiguous()
        if T * topk <= SHARED_FUSED_MAX_PAIRS and H % 512 == 0 and I % 512 == 0:
            _lib.call("d3_moe_fp8_forward_shared", _lib.ptr(x), _lib.ptr(ids),
                      ids.element_size(), _lib.ptr(weights), wf, T, topk, _lib.ptr(w13),
                      _lib.ptr(s13), _lib.ptr(w2), _lib.ptr(s2), n, H, I, _lib.ptr(sw13),
                      _lib.ptr(sw2), _lib.ptr(sg) if sg is not None else None, _lib.ptr(out),
                      1 if accumulate else 0, _lib.ptr(error_word(dev)), _lib.ptr(ws),
                      ws.numel(), _lib.stream_ptr(stream))
            return out
        # larger batches: the routed experts, then the shared expert as two
        # plain bf16 GEMMs (library GEMMs) added in fp32
        y = torch.nn.functional.linear(x, sw13).float()
        hs = torch.nn.functional.silu(y[:, :I]) * y[:, I:]
        ys = torch.nn.functional.linear(hs.to(torch.bfloat16), sw2).float()
        if sg is not None:
            ys = ys * torch.sigmoid(x.float() @ sg.float())[:, None]
        base = out.float() if accumulate else torch.zeros_like(ys)
        fp8_moe_forward(x, ids, weights, w13, s13, w2, s2, out=out, accumulate=False,
                        stream=stream)
        out.copy_((base + out.float() + ys).to(torch.bfloat16))
        return out
    _lib.call("d3_moe_fp8_forward", _lib.ptr(x), _lib.ptr(ids), ids.element_size(),
              _lib.ptr(weights), wf, T, topk,
              _lib.ptr(w13), _lib.ptr(s13), _lib.ptr(w2), _lib.ptr(s2), n, H, I, _lib.ptr(out),
              1 if accumulate else 0, _lib.ptr(error_word(dev)), _lib.ptr(ws), ws.numel(),
              _lib.stream_ptr(stream))
    return out


def fp8_moe_forward_p2p(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                        w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor,
                        s2: torch.Tensor, *, wait_flags: torch.Tensor, epoch: torch.Tensor,
                        n_ranks: int, rank: int, cap: int, peer_ret, peer_flag_r,
                        counter: torch.Tensor, wait_code: int, budget_ns: int,
                        stream=None) -> None:
    """The expert call of one expert-parallel layer over NVLink peer memory
    (``d3_moe_fp8_forward_p2p``): waits for every source's dispatch epoch in
    ``wait_flags``, runs the routed experts on the received rows ``x``
    ([n_ranks * cap, H] bf16, ids = local expert ids, -1 for unused rows) and
    stores each served row straight into its source's return buffer
    (``peer_ret``: ctypes array of n_ranks device pointers), publishing the
    epoch in every source's flag_r (``peer_flag_r``).  Nothing is returned
    locally."""
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise TypeError("x must be contiguous bf16")
    T, H = x.shape
    ids = ids.reshape(T, -1)
    topk = ids.shape[1]
    if ids.dtype not in (torch.int32, torch.int64) or not ids.is_contiguous():
        raise TypeError("ids must be contiguous int32/int64")
    weights = weights.reshape(T, topk)
    if weights.dtype not in (torch.float32, torch.bfloat16) or not weights.is_contiguous():
        raise TypeError("weights must be contiguous f32/bf16")
    n, two_i, h2 = w13.shape
    if h2 != H or w2.shape[0] != n or w2.shape[1] != H:
        raise ValueError("weight shapes do not match x")
    I = two_i // 2
    dev = x.device
    need = workspace_bytes(T, topk, n, H, I)
    if need == 0:
        raise ValueError(f"unsupported MoE shape T={T} topk={topk} n={n} H={H} I={I}")
    ws = _workspace(dev, need, "moe")
    wf = 1 if weights.dtype == torch.float32 else 0
    _lib.call("d3_moe_fp8_forward_p2p", _lib.ptr(x), _lib.ptr(ids), ids.element_size(),
              _lib.ptr(weights), wf, T, topk, _lib.ptr(w13), _lib.ptr(s13), _lib.ptr(w2),
              _lib.ptr(s2), n, H, I, _lib.ptr(error_word(dev)), _lib.ptr(ws), ws.numel(),
              _lib.ptr(wait_flags), _lib.ptr(epoch), n_ranks, rank, cap, peer_ret, peer_flag_r,
              _lib.ptr(counter), wait_code, budget_ns, _lib.stream_ptr(stream))
