"""The C-ABI library builds, loads and exports every declared symbol (no GPU).

Only argument validation is exercised here: those paths return before any
CUDA call, so they run on a machine without a GPU.
"""
import ctypes
import re
from pathlib import Path

import pytest

from drama3_offloading_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "d3b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^D3_API\s+[\w\s\*]+?\b(d3_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_bound_set():
    decl = declared_functions()
    assert len(decl) == len(set(decl)) and decl
    assert set(decl) == set(_lib.SIGNATURES), (set(decl) ^ set(_lib.SIGNATURES))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.d3_abi_version() >= 1


def test_status_strings():
    lib = _lib.load()
    for code, name in _lib.STATUS.items():
        assert lib.d3_status_string(code).decode() == name


def test_argument_validation_without_gpu():
    lib = _lib.load()
    P = ctypes.c_void_p
    # misaligned expert size -> D3_ERR_MISALIGNED, message names the problem
    rc = lib.d3_fetch_experts(P(16), P(16), P(16), P(16), P(16), 24, 1, 1, 256, P(0))
    assert rc == -3 and b"16" in lib.d3_last_error()
    # threads other than 256 -> invalid argument
    rc = lib.d3_fetch_experts(P(16), P(16), P(16), P(16), P(16), 32, 1, 1, 128, P(0))
    assert rc == -1
    # null pointers
    assert lib.d3_fetch_experts(P(0), P(16), P(16), P(16), P(16), 32, 1, 1, 256, P(0)) == -1
    # resolve: k out of range, capacity too large
    z = P(16)
    assert lib.d3_resolve_slots(z, 4, 0, z, 8, z, z, 4, z, z, z, z, z, P(0)) == -1
    assert lib.d3_resolve_slots(z, 4, 8, z, 8, z, z, 9000, z, z, z, z, z, P(0)) == -6
    assert lib.d3_resolve_slots(z, 3, 8, z, 8, z, z, 4, z, z, z, z, z, P(0)) == -1
    # fused resolve+fetch: descriptor checks
    d = _lib.LayerCache()
    d.num_experts, d.capacity, d.policy, d.nbuf = 8, 4, 0, 5
    assert lib.d3_resolve_fetch(ctypes.byref(d), z, 4, 8, 0, P(0)) == -1
    d.nbuf = 1
    for n in ("slot_of", "slot_expert", "stamp", "step", "out_slot", "fetch_slot",
              "fetch_expert", "nmiss"):
        setattr(d, n, 16)
    d.host[0], d.cache[0], d.bytes[0] = 16, 16, 40
    assert lib.d3_resolve_fetch(ctypes.byref(d), z, 4, 8, 0, P(0)) == -3
    d.policy = 1  # LFU without freq/ins tables
    d.bytes[0] = 48
    assert lib.d3_resolve_fetch(ctypes.byref(d), z, 4, 8, 0, P(0)) == -1
    # census / trace: null pointers, id width, a call larger than the ring
    assert lib.d3_census_add(P(0), 4, 1, 8, 256, z, z, P(0)) == -1
    assert lib.d3_census_add(z, 2, 1, 8, 256, z, z, P(0)) == -1
    assert lib.d3_trace_append(z, 4, 10, 8, 0, z, z, 4, P(0)) == -6
    assert lib.d3_trace_append(z, 4, 1, 8, 0, P(0), z, 4, P(0)) == -1


def test_folded_entry_points_validate_without_gpu():
    """The overlapped decode call and the folded NVLink expert-parallel calls
    reject bad shapes and descriptors before touching the GPU."""
    lib = _lib.load()
    P = ctypes.c_void_p
    z = P(16)
    I64 = ctypes.c_int64
    # d3_resolve_fetch_moe: workspace size, shape, buffer layout, capacity < k
    assert lib.d3_resolve_fetch_moe_workspace_size(8, 2048, 512) >= 512 + 4 * (8 * 512 + 513)
    assert lib.d3_resolve_fetch_moe_workspace_size(0, 2048, 512) == 0
    d = _lib.LayerCache()
    d.num_experts, d.capacity, d.policy, d.nbuf = 64, 12, 0, 4
    sizes = (2 * 512 * 2048, 2048 * 512, 8 * 16 * 4, 16 * 4 * 4)
    for b, n in enumerate(sizes):
        d.host[b], d.cache[b], d.bytes[b] = 16, 16, n
    ws = ctypes.c_size_t(1 << 20)
    call = lambda desc, k, H, I, wsz: lib.d3_resolve_fetch_moe(
        ctypes.byref(desc), z, 4, k, z, z, 1, H, I, None, None, None, z, 0, z, z, wsz, 0, 3, P(0))
    assert call(d, 8, 2048, 384, ws) == -5          # I not a multiple of 512
    d.bytes[1] = 1234
    assert call(d, 8, 2048, 512, ws) == -1          # buffer sizes do not match H, I
    d.bytes[1] = sizes[1]
    d.capacity = 4
    assert call(d, 8, 2048, 512, ws) == -5          # capacity < k
    d.capacity = 12
    assert call(d, 8, 2048, 512, ctypes.c_size_t(64)) == -7   # workspace too small
    d.nbuf = 3
    assert call(d, 8, 2048, 512, ws) == -1          # not the 4-buffer layout
    d.nbuf = 4
    # d3_resolve_fetch_moe_l2warm: the window list, then the same checks
    ptrs = (P * 5)(16, 16, 16, 16, 16)
    nbs = (ctypes.c_size_t * 5)(1 << 20, 4096, 128, 0, 7)
    warm = lambda desc, k, pp, nn, n: lib.d3_resolve_fetch_moe_l2warm(
        ctypes.byref(desc), z, 4, k, z, z, 1, 2048, 512, None, None, None, z, 0, z, z, ws, 0, 3,
        pp, nn, n, P(0))
    assert warm(d, 8, ptrs, nbs, 5) == -1           # more than 4 windows
    assert warm(d, 8, None, None, 2) == -1          # null window arrays
    assert warm(d, 8, ptrs, nbs, -1) == -1
    nulls = (P * 2)(16, 0)
    assert warm(d, 8, nulls, nbs, 2) == -1          # null window with bytes
    d.capacity = 4
    assert warm(d, 8, ptrs, nbs, 4) == -5           # then the plain call's checks: capacity < k
    assert b"capacity" in lib.d3_last_error()
    d.capacity = 12
    # d3_moe_fp8_forward_p2p: T must be n_ranks * cap, ranks in range
    arr = (P * 2)(16, 16)
    p2p = lambda T, n_ranks, rank, cap: lib.d3_moe_fp8_forward_p2p(
        z, z, 4, z, 1, T, 1, z, z, z, z, 32, 2048, 512, z, z, ctypes.c_size_t(1 << 20), z, z,
        n_ranks, rank, cap, arr, arr, z, 31, I64(10**9), P(0))
    assert p2p(100, 2, 0, 64) == -1
    assert p2p(128, 2, 2, 64) == -1
    assert p2p(128, 17, 0, 64) == -6
    # d3_ep_combine_p2p: rank count and wait budget
    comb = lambda n_ranks, budget: lib.d3_ep_combine_p2p(
        z, z, z, 1, 8, 8, 2048, z, 0, z, n_ranks, z, z, 32, I64(budget), P(0))
    assert comb(0, 10**9) == -6
    assert comb(2, 0) == -1


def test_layer_cache_struct_layout():
    # 4 int32, 11 pointers, 4+4 pointers, 4 int64
    assert ctypes.sizeof(_lib.LayerCache) == 16 + 11 * 8 + 8 * 8 + 4 * 8


def test_device_error_codes_are_named():
    """Every code a kernel writes into the device error word has a message."""
    from drama3_offloading_b200 import moe
    src = (Path(__file__).resolve().parent.parent / "drama3_offloading_b200" / "csrc")
    text = "".join(f.read_text() for f in sorted(src.glob("*.cu*")))
    codes = {int(c) for c in re.findall(r"gemm_error\(p\.err, (\d+)\)", text)}
    codes |= {int(c) for c in re.findall(r"err_code = (\d+)", text)}
    codes |= {int(c) for c in re.findall(r"kFusedBarrierCode = (\d+)", text)}
    codes |= {31, 32}   # the expert-parallel waits' codes, passed in by ep.py
    assert codes and codes <= set(moe.ERROR_CODES), codes - set(moe.ERROR_CODES)
    assert moe.error_message(999) == "unknown bounded wait"
