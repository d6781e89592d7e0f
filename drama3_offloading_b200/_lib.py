"""ctypes binding of libd3b200.so (declarations: include/d3b200.h).

The library is built in-tree by ``drama3_offloading_b200.build``.  There is no
fallback: if the shared library is missing or fails to load, every entry point
raises, so a GPU run can never silently compute on another path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libd3b200.so"

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
SZ = ctypes.c_size_t

D3_OK = 0
STATUS = {0: "D3_OK", -1: "D3_ERR_INVALID_ARG", -2: "D3_ERR_NOT_PINNED", -3: "D3_ERR_MISALIGNED",
          -4: "D3_ERR_CUDA", -5: "D3_ERR_UNSUPPORTED", -6: "D3_ERR_TOO_LARGE",
          -7: "D3_ERR_WORKSPACE"}
D3_POLICY_LRU, D3_POLICY_LFU = 0, 1
D3_MAX_BUFFERS = 4


class D3Error(RuntimeError):
    def __init__(self, status: int, func: str, msg: str):
        self.status = status
        super().__init__(f"{func} -> {STATUS.get(status, status)}: {msg}")


class LayerCache(ctypes.Structure):
    """Mirror of ``d3_layer_cache`` (include/d3b200.h)."""
    _fields_ = [
        ("num_experts", I32), ("capacity", I32), ("policy", I32), ("nbuf", I32),
        ("slot_of", P), ("slot_expert", P), ("stamp", P), ("step", P),
        ("freq", P), ("ins", P), ("out_slot", P), ("fetch_slot", P),
        ("fetch_expert", P), ("nmiss", P), ("counters", P),
        ("host", P * D3_MAX_BUFFERS), ("cache", P * D3_MAX_BUFFERS),
        ("bytes", I64 * D3_MAX_BUFFERS),
    ]


# name -> (restype, argtypes); every function declared in include/d3b200.h
SIGNATURES: dict[str, tuple] = {
    "d3_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "d3_last_error": (ctypes.c_char_p, []),
    "d3_abi_version": (ctypes.c_int, []),
    "d3_device_ptr_of": (ctypes.c_int, [P, SZ, ctypes.POINTER(P)]),
    "d3_fetch_experts": (ctypes.c_int, [P, P, P, P, P, I64, I32, I32, I32, P]),
    "d3_resolve_slots": (ctypes.c_int, [P, I32, I32, P, I32, P, P, I32, P, P, P, P, P, P]),
    "d3_resolve_fetch": (ctypes.c_int, [ctypes.POINTER(LayerCache), P, I32, I32, I32, P]),
    "d3_lookup_slots": (ctypes.c_int, [P, I32, P, I32, I32, P, P]),
    "d3_fetch_jobs": (ctypes.c_int, [ctypes.POINTER(LayerCache), I32, P]),
    "d3_router_workspace_size": (SZ, [I32, I32]),
    "d3_router_topk": (ctypes.c_int, [P, P, I32, I32, I32, I32, I32, P, P, P, P, SZ, P]),
    "d3_router_topk_noalloc": (ctypes.c_int, [P, P, I32, I32, I32, I32, I32, P, P, P, P]),
    "d3_moe_workspace_size": (SZ, [I32, I32, I32, I32, I32]),
    "d3_moe_fp8_forward": (ctypes.c_int, [P, P, I32, P, I32, I32, I32, P, P, P, P, I32, I32,
                                          I32, P, I32, P, P, SZ, P]),
    "d3_moe_fp8_forward_shared": (ctypes.c_int, [P, P, I32, P, I32, I32, I32, P, P, P, P, I32,
                                                 I32, I32, P, P, P, P, I32, P, P, SZ, P]),
    "d3_prefill_plan": (ctypes.c_int, [P, I32, I32, I32, P, P, P, P, P]),
    "d3_gather_experts": (ctypes.c_int, [ctypes.POINTER(LayerCache), P, P, P, P, I32, P]),
    "d3_ep_dispatch_pack":(ctypes.c_int, [P, P, I32, I32, I32, I32, I32, I32, P, P, P, P, P]),
    "d3_ep_combine": (ctypes.c_int, [P, P, P, I32, I32, I32, I32, P, I32, P]),
    "d3_ipc_get": (ctypes.c_int, [P, P, P]),
    "d3_ipc_open": (ctypes.c_int, [P, P]),
    "d3_ipc_close": (ctypes.c_int, [P]),
    "d3_ep_dispatch_p2p": (ctypes.c_int, [P, P, I32, I32, I32, I32, I32, I32, I32, P, P, P, P, P,
                                          P, P, P]),
    "d3_ep_return_p2p": (ctypes.c_int, [P, P, I32, I32, I32, I32, P, P, P, P, P]),
    "d3_ep_wait": (ctypes.c_int, [P, I32, P, P, I32, I64, P]),
    "d3_resolve_fetch_moe_workspace_size": (SZ, [I32, I32, I32]),
    "d3_resolve_fetch_moe": (ctypes.c_int, [ctypes.POINTER(LayerCache), P, I32, I32, P, P, I32,
                                            I32, I32, P, P, P, P, I32, P, P, SZ, I32, I32, P]),
    "d3_resolve_fetch_moe_l2warm": (ctypes.c_int, [ctypes.POINTER(LayerCache), P, I32, I32, P, P,
                                                   I32, I32, I32, P, P, P, P, I32, P, P, SZ, I32,
                                                   I32, P, P, I32, P]),
    "d3_moe_fp8_forward_p2p": (ctypes.c_int, [P, P, I32, P, I32, I32, I32, P, P, P, P, I32, I32,
                                              I32, P, P, SZ, P, P, I32, I32, I32, P, P, P, I32,
                                              I64, P]),
    "d3_ep_combine_p2p": (ctypes.c_int, [P, P, P, I32, I32, I32, I32, P, I32, P, I32, P, P, I32,
                                         I64, P]),
    "d3_census_add": (ctypes.c_int, [P, I32, I32, I32, I32, P, P, P]),
    "d3_trace_append": (ctypes.c_int, [P, I32, I32, I32, I32, P, P, I64, P]),
}

_lib = None
_load_error: str | None = None


def load() -> ctypes.CDLL:
    """Load the library (building it first if it is absent and nvcc exists)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() and os.environ.get("D3_NO_AUTOBUILD") is None:
        try:
            from . import build as _build
            _build.build()
        except Exception as exc:  # reported below
            _load_error = f"build failed: {exc}"
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        _load_error = f"cannot load {LIB_PATH}: {exc}" + (f" ({_load_error})" if _load_error else "")
        raise RuntimeError(_load_error) from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    if _lib is None:
        return _load_error or ""
    return _lib.d3_last_error().decode()


def call(name: str, *args) -> None:
    """Call ``name`` and raise D3Error on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != D3_OK:
        raise D3Error(rc, name, lib.d3_last_error().decode())


def ptr(t) -> P:
    """Raw data pointer of a torch tensor (or None)."""
    return P(0) if t is None else P(t.data_ptr())


def stream_ptr(stream=None) -> P:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return P(s.cuda_stream)
