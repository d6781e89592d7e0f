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


def test_layer_cache_struct_layout():
    # 4 int32, 11 pointers, 4+4 pointers, 4 int64
    assert ctypes.sizeof(_lib.LayerCache) == 16 + 11 * 8 + 8 * 8 + 4 * 8
