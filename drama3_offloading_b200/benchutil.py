"""Measurement helpers shared by bench.py: host-link peak, clock sampling,
CUDA-event timing and distributed plumbing."""
from __future__ import annotations

import csv
import io
import os
import statistics
import subprocess
import tempfile
import time

import torch

GiB = 1 << 30


def host_link_peak_gbs(nbytes: int = GiB, reps: int = 8, device=None) -> dict:
    """Best-of-N pinned host->device copy-engine bandwidth (GB/s, 1e9 B/s) of a
    >= 1 GiB buffer: the roofline for any host->device fetch on this box
    (bin/bench_pin.py:28-61 / bin/bench_hostread.py MemcpyBaseline method)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    src.fill_(1)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize(device)
    best = 0.0
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b)
        times.append(ms)
        best = max(best, nbytes / (ms * 1e-3) / 1e9)
    del src, dst
    return {"gbs": best, "bytes": nbytes, "reps": reps, "ms": times}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while active."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int | None = None):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="d3clk_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
               "-lms", "200"]
        if self.index is not None:
            cmd += ["-i", str(self.index)]
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        with open(self.path) as f:
            for r in csv.reader(f):
                if len(r) >= 9:
                    rows.append([c.strip() for c in r])
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_env() -> tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int, device=None) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index] if device is not None else None)
