"""The allocation-free router entry point, d3_router_topk_noalloc.

It exists for callers that cannot allocate device memory -- a runtime that
binds only the C ABI and has no device allocator, a decode loop that must
never allocate, a process whose free device memory all went to the expert
cache -- so its scratch lives in a fixed array inside the library.  Here it is
called through the C ABI and must give the same ids (exactly) and weights
(within the tolerance the router tests use) as d3_router_topk with a caller
workspace, on two calls in a row (the shared scratch must come back clean),
and it must reject a size beyond its fixed scratch with D3_ERR_TOO_LARGE.

The file name sorts last so a run that stops at the first failure has run
every other test first; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from drama3_offloading_b200 import _lib  # noqa: E402

DEV = torch.device("cuda:0")
P = ctypes.c_void_p


def _with_workspace(x, gw, k):
    T, H = x.shape
    E = gw.shape[0]
    lib = _lib.load()
    ws = torch.zeros(lib.d3_router_workspace_size(T, E), dtype=torch.uint8, device=DEV)
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=DEV)
    _lib.call("d3_router_topk", P(x.data_ptr()), P(gw.data_ptr()), T, H, E, k, 1,
              P(ids.data_ptr()), P(w.data_ptr()), P(0), P(ws.data_ptr()), ws.numel(),
              _lib.stream_ptr())
    return ids, w


def _noalloc(x, gw, k):
    T, H = x.shape
    E = gw.shape[0]
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=DEV)
    wb = torch.empty(T, k, dtype=torch.bfloat16, device=DEV)
    _lib.call("d3_router_topk_noalloc", P(x.data_ptr()), P(gw.data_ptr()), T, H, E, k, 1,
              P(ids.data_ptr()), P(w.data_ptr()), P(wb.data_ptr()), _lib.stream_ptr())
    return ids, w, wb


def test_noalloc_router_matches_workspace_router_twice():
    """Every router kernel through the fixed scratch, calls back to back:
    T = 1, 2 (the cluster kernel, no scratch), 3 and 16 (4-warp split), 64
    (unsplit general kernel) and 256 at E = 256 (T * E = 65536: the logits
    fill the whole array, its last element included), then T = 16 again.
    Each call must equal the workspace router (ids exactly, weights within
    the router tests' tolerance) and the CPU oracle's ids and weights."""
    g = torch.Generator().manual_seed(99)
    gw_c = (torch.randn(256, 2048, generator=g) * 0.02).to(torch.bfloat16)
    gw = gw_c.to(DEV)
    for T in (1, 2, 3, 16, 64, 256, 16):
        x_c = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
        x = x_c.to(DEV)
        want_ids, want_w = _with_workspace(x, gw, 8)
        ids, w, wb = _noalloc(x, gw, 8)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.cpu().numpy(), want_ids.cpu().numpy())
        np.testing.assert_allclose(w.cpu().numpy(), want_w.cpu().numpy(), rtol=1e-5, atol=1e-7)
        np.testing.assert_array_equal(wb.float().cpu().numpy(),
                                      want_w.to(torch.bfloat16).float().cpu().numpy())
        ref_ids, ref_w, _, _ = oracle.router_topk(x_c, gw_c, 8)
        np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids.numpy())
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.numpy(), rtol=1e-5, atol=1e-7)


def test_noalloc_router_rejects_oversize():
    gw = torch.zeros(256, 2048, dtype=torch.bfloat16, device=DEV)
    x = torch.zeros(512, 2048, dtype=torch.bfloat16, device=DEV)  # 512*256 > 65536
    ids = torch.empty(512, 8, dtype=torch.int32, device=DEV)
    rc = _lib.load().d3_router_topk_noalloc(P(x.data_ptr()), P(gw.data_ptr()), 512, 2048, 256,
                                            8, 1, P(ids.data_ptr()), P(0), P(0),
                                            _lib.stream_ptr())
    assert rc == -6  # D3_ERR_TOO_LARGE
    assert b"scratch" in _lib.load().d3_last_error()
