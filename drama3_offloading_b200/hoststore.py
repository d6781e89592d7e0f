"""One page-locked copy of the offloaded expert bytes per machine, shared by
every local rank.

The reference keeps all 30 GiB of routed experts in pinned host RAM for its one
GPU (bin/offload.py:664-699 pin_experts).  With one process per GPU, a private
copy per rank would need 8 x 30 GiB on an 8-GPU box -- more RAM than the box
has.  Here local rank 0 creates an anonymous shared-memory file (memfd) of the
store's size and fills it; the other local ranks open the same file through
/proc/<pid>/fd/<fd>, map it, and every rank page-locks and device-maps its
mapping with cudaHostRegister(PORTABLE | MAPPED), so each GPU's fetch kernel
reads the one copy over its own PCIe link.

Before allocating, the free RAM is checked (MemAvailable); a store that does
not fit raises MemoryError instead of driving the host out of memory.
"""
from __future__ import annotations

import mmap
import os

import torch

GiB = 1 << 30
_REGISTER_PORTABLE_MAPPED = 1 | 2   # cudaHostRegisterPortable | cudaHostRegisterMapped
_CHUNK = 1 << 30


def mem_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def _align(v: int, a: int = 4096) -> int:
    return (v + a - 1) // a * a


class SharedHostStore:
    """``nbytes`` of shared, page-locked, device-mapped host memory.

    ``group``: torch.distributed process group of the ranks on this machine
    (None for a single process).  ``local_rank`` 0 creates and owns the file."""

    def __init__(self, nbytes: int, local_rank: int = 0, group=None, headroom: int = 8 * GiB):
        import torch.distributed as dist
        self.nbytes = nbytes = _align(nbytes)
        self.owner = local_rank == 0
        multi = group is not None and dist.is_initialized() and dist.get_world_size(group) > 1
        info = [None]
        err = None
        if self.owner:
            avail = mem_available()
            if avail and nbytes + headroom > avail:
                err = (f"shared expert store needs {nbytes / GiB:.1f} GiB + {headroom / GiB:.0f} "
                       f"GiB headroom, only {avail / GiB:.1f} GiB available")
            else:
                fd = os.memfd_create("d3_expert_store", 0)
                os.ftruncate(fd, nbytes)
                self.fd = fd
                info = [(os.getpid(), fd)]
        if multi:
            payload = [err if err else info[0]]
            dist.broadcast_object_list(payload, src=dist.get_global_rank(group, 0), group=group)
            if isinstance(payload[0], str):
                err = payload[0]
            else:
                info = payload
        if err:
            raise MemoryError(err)
        if not self.owner:
            pid, fd = info[0]
            self.fd = os.open(f"/proc/{pid}/fd/{fd}", os.O_RDWR)
        self.mm = mmap.mmap(self.fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.buf = torch.frombuffer(self.mm, dtype=torch.uint8)
        self.chunks = []
        self.regions = []          # (offset, bytes) of every take(), registered one by one
        self.registered = False
        self._off = 0

    def register(self) -> None:
        """Page-lock and device-map every region handed out by take(), each as
        its own registration of at most 1 GiB.  Per-region registration keeps
        every tensor inside one registration (a copy into a tensor spanning two
        is rejected), and several processes registering one huge range of
        not-yet-faulted shared pages at the same time was refused by the OS
        (cudaErrorOperatingSystem) on this pool while piecewise registration of
        the same bytes was not.  Call it on the owner before filling, on the
        other ranks after the owner's fill."""
        if self.registered:
            return
        rt = torch.cuda.cudart()
        base = self.buf.data_ptr()
        for off0, nb in self.regions:
            for off in range(off0, off0 + nb, _CHUNK):
                n = min(_CHUNK, off0 + nb - off)
                rc = int(rt.cudaHostRegister(base + off, n, _REGISTER_PORTABLE_MAPPED))
                if rc != 0:
                    self.close()
                    raise RuntimeError(f"cudaHostRegister of the shared expert store failed "
                                       f"(cudaError {rc}) at offset {off}")
                self.chunks.append(base + off)
        self.registered = True

    def take(self, shape, dtype) -> torch.Tensor:
        """Next page-aligned sub-tensor of the store."""
        n = 1
        for s in shape:
            n *= s
        nb = n * torch.empty((), dtype=dtype).element_size()
        if self._off + nb > self.nbytes:
            raise ValueError("shared store exhausted")
        t = self.buf[self._off:self._off + nb].view(dtype).view(*shape)
        self.regions.append((self._off, nb))
        self._off = _align(self._off + nb)
        return t

    def close(self) -> None:
        """Unregister every chunk.  Must run before the mapping goes away: a
        registration left behind after the pages are unmapped makes later
        copies into host memory that reuses those addresses fail."""
        rt = torch.cuda.cudart() if getattr(self, "chunks", None) else None
        for p in getattr(self, "chunks", []):
            rt.cudaHostUnregister(p)
        self.chunks = []
        self.registered = False

    def __del__(self):
        # self.mm (the mapping) is released only after this runs
        try:
            self.close()
        except Exception:
            pass


def layer_bytes(E: int, H: int, I: int) -> int:
    return (_align(E * 2 * I * H) + _align(E * H * I) + _align(E * (2 * I // 128) * (H // 128) * 4)
            + _align(E * (H // 128) * (I // 128) * 4))
