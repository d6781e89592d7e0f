"""Synthetic expert weights in the Drama-3 layout (random init; no checkpoint).

Runtime layout per MoE layer (bin/offload.py:111-134, notes/01-static-findings.md:93-97):
``w13_weight [E, 2I, H]`` e4m3 (gate rows [0, I), up rows [I, 2I)),
``w2_weight [E, H, I]`` e4m3, ``w13_scale_inv [E, 2I/128, H/128]`` f32,
``w2_scale_inv [E, H/128, I/128]`` f32 -- 3,146,496 bytes per expert at
H=2048, I=512.

``HostExperts`` stands in for upstream ``MoEExperts`` (absent here): it
carries exactly the attributes the device cache reads.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

BLOCK = 128


@dataclass
class HostExperts:
    num_experts: int
    w13_weight: torch.Tensor
    w2_weight: torch.Tensor
    w13_scale_inv: torch.Tensor
    w2_scale_inv: torch.Tensor

    def pin(self) -> "HostExperts":
        for n in ("w13_weight", "w2_weight", "w13_scale_inv", "w2_scale_inv"):
            t = getattr(self, n)
            if t.device.type == "cpu" and not t.is_pinned():
                setattr(self, n, t.pin_memory())
        return self

    def to(self, device) -> "HostExperts":
        return HostExperts(self.num_experts, *(getattr(self, n).to(device) for n in (
            "w13_weight", "w2_weight", "w13_scale_inv", "w2_scale_inv")))


def quantize_blocks(w: torch.Tensor):
    """fp32 [..., R, C] -> (e4m3, f32 scale_inv [..., R/128, C/128]): per 128x128
    block ``scale_inv = amax / 448`` and ``q = e4m3(w / scale_inv)``."""
    *lead, R, C = w.shape
    rb, cb = R // BLOCK, C // BLOCK
    blk = w.reshape(*lead, rb, BLOCK, cb, BLOCK)
    amax = blk.abs().amax(dim=(-3, -1))
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (blk / s[..., :, None, :, None]).reshape(*lead, R, C)
    return q.to(torch.float8_e4m3fn), s.to(torch.float32)


def make_experts(E: int, H: int = 2048, I: int = 512, seed: int = 0, device="cpu",
                 style: str = "normal", chunk: int = 16) -> HostExperts:
    """Random expert weights.

    ``style="normal"``: weights N(0, 0.02) quantised per 128x128 block
    (the single-layer configuration).  ``style="test"``: the reference test's
    construction, ``randn*0.2 -> e4m3`` with scales ``rand*0.1+0.05``
    (bin/test_devcache.py:33-37).  Generated in chunks of ``chunk`` experts on
    ``device`` with a seeded generator.
    """
    g = torch.Generator(device=device).manual_seed(seed)
    w13 = torch.empty(E, 2 * I, H, dtype=torch.float8_e4m3fn, device=device)
    w2 = torch.empty(E, H, I, dtype=torch.float8_e4m3fn, device=device)
    s13 = torch.empty(E, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=device)
    s2 = torch.empty(E, H // BLOCK, I // BLOCK, dtype=torch.float32, device=device)
    for lo in range(0, E, chunk):
        hi = min(E, lo + chunk)
        n = hi - lo
        if style == "normal":
            a = torch.randn(n, 2 * I, H, generator=g, device=device) * 0.02
            w13[lo:hi], s13[lo:hi] = quantize_blocks(a)
            del a
            b = torch.randn(n, H, I, generator=g, device=device) * 0.02
            w2[lo:hi], s2[lo:hi] = quantize_blocks(b)
            del b
        elif style == "test":
            w13[lo:hi] = (torch.randn(n, 2 * I, H, generator=g, device=device) * 0.2).to(
                torch.float8_e4m3fn)
            w2[lo:hi] = (torch.randn(n, H, I, generator=g, device=device) * 0.2).to(
                torch.float8_e4m3fn)
            s13[lo:hi] = torch.rand(n, 2 * I // BLOCK, H // BLOCK, generator=g, device=device) * 0.1 + 0.05
            s2[lo:hi] = torch.rand(n, H // BLOCK, I // BLOCK, generator=g, device=device) * 0.1 + 0.05
        else:
            raise ValueError(style)
    return HostExperts(E, w13, w2, s13, s2)


def pattern_experts(E: int, H: int = 2048, I: int = 512, pin: bool = True) -> HostExperts:
    """Self-identifying bytes (bin/bench_hostread.py:257-292): int64 element k of
    expert e in buffer b is ``(b << 56) | (e << 32) | k``, so a byte in the
    wrong slot, at the wrong offset or from the wrong buffer is detectable."""
    shapes = [((E, 2 * I, H), torch.float8_e4m3fn), ((E, H, I), torch.float8_e4m3fn),
              ((E, 2 * I // BLOCK, H // BLOCK), torch.float32),
              ((E, H // BLOCK, I // BLOCK), torch.float32)]
    out = []
    for b, (shape, dt) in enumerate(shapes):
        t = torch.empty(shape, dtype=dt, pin_memory=pin)
        v = t.view(torch.uint8).reshape(E, -1).view(torch.int64)
        k = torch.arange(v.shape[1], dtype=torch.int64)
        for e in range(E):
            torch.add(k, (b << 56) | (e << 32), out=v[e])
        out.append(t)
    return HostExperts(E, *out)


def pattern_expected(b: int, e: int, n64: int) -> torch.Tensor:
    return torch.arange(n64, dtype=torch.int64) + ((b << 56) | (e << 32))
