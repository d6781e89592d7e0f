"""Page-locked copies of the offloaded expert bytes shared by the local
ranks of a machine: one copy per NUMA node that holds one of the ranks' GPUs.

The reference keeps all 30 GiB of routed experts in pinned host RAM for its one
GPU (bin/offload.py:664-699 pin_experts).  With one process per GPU, a private
copy per rank would need 8 x 30 GiB on an 8-GPU box -- more RAM than the box
has -- and one copy for all ranks puts every GPU's expert reads on the DRAM of
one node (and, for the GPUs attached to the other socket, on the inter-socket
link).  Here the lowest local rank of each NUMA node creates an anonymous
shared-memory file (memfd) of the store's size, sets its pages' placement to
that node (mbind, MPOL_PREFERRED) before they are first touched, and fills it
(local rank 0 from the generator, the other nodes' owners by copying local
rank 0's bytes); the other local ranks open their node's file through
/proc/<pid>/fd/<fd> and map it.  Every rank page-locks and device-maps its
mapping with cudaHostRegister(PORTABLE | MAPPED), so each GPU's fetch kernel
reads a copy on its own node over its own PCIe link.  Every copy holds the
same bytes.

One copy for all ranks (the placement left to the kernel) when the GPUs'
nodes are unknown (sysfs reports -1), all on one node, or when a node has no
room for a copy; a single rank binds its copy to its GPU's node.  Before
allocating, the free RAM is checked (MemAvailable, and each node's MemFree
for per-node copies); a store that does not fit raises MemoryError instead of
driving the host out of memory.
"""
from __future__ import annotations

import ctypes
import mmap
import os
import platform

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


def gpu_numa_node(device) -> int:
    """NUMA node of the GPU's PCI function as sysfs reports it; -1 when the
    platform does not say (no NUMA, a virtual machine, no sysfs)."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            return max(-1, int(f.read().strip()))
    except (AttributeError, OSError, ValueError, RuntimeError, AssertionError):
        return -1


def node_mem_free(node: int) -> int:
    """Free bytes of NUMA node ``node`` (0 when unknown)."""
    if node < 0:
        return 0
    try:
        with open(f"/sys/devices/system/node/node{node}/meminfo") as f:
            for line in f:
                if "MemFree:" in line:
                    return int(line.split()[-2]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return 0


_MPOL_PREFERRED = 1
_SYS_MBIND = {"x86_64": 237, "aarch64": 235}


def bind_to_node(addr: int, length: int, node: int) -> bool:
    """Place the not-yet-touched pages of [addr, addr + length) on ``node``
    (mbind, MPOL_PREFERRED: the node's memory while it has room, any other
    node's after).  For a shared-memory mapping the policy belongs to the
    file, so it holds for every process that maps it.  False when the
    platform refuses it (no NUMA support, a seccomp filter); the pages are
    then placed by the default policy."""
    nr = _SYS_MBIND.get(platform.machine())
    if nr is None or node < 0 or node >= 1024:
        return False
    mask = (ctypes.c_ulong * 16)()
    mask[node // 64] = 1 << (node % 64)
    libc = ctypes.CDLL(None, use_errno=True)
    libc.syscall.restype = ctypes.c_long
    rc = libc.syscall(ctypes.c_long(nr), ctypes.c_long(addr), ctypes.c_long(length),
                      ctypes.c_long(_MPOL_PREFERRED), mask, ctypes.c_long(1025), ctypes.c_long(0))
    return rc == 0


class SharedHostStore:
    """``nbytes`` of shared, page-locked, device-mapped host memory.

    ``group``: torch.distributed process group of the ranks on this machine
    (None for a single process).  ``node``: the NUMA node of this rank's GPU
    (``gpu_numa_node``; -1 unknown).  With ``per_node`` and the ranks' GPUs on
    more than one known node, each node gets its own copy, created by the
    lowest local rank on it (``owner``); otherwise local rank 0 creates the
    one copy.  ``primary`` (local rank 0) fills its copy; the other owners
    take theirs from it with ``copy_from_primary``."""

    _NODE_HEADROOM = 4 * GiB

    def __init__(self, nbytes: int, local_rank: int = 0, group=None, headroom: int = 8 * GiB,
                 node: int = -1, per_node: bool = True):
        import torch.distributed as dist
        self.nbytes = nbytes = _align(nbytes)
        multi = group is not None and dist.is_initialized() and dist.get_world_size(group) > 1
        self.primary = local_rank == 0 or not multi
        if not multi:
            local_rank = 0

        def gather(obj):
            if not multi:
                return [obj]
            out = [None] * dist.get_world_size(group)
            dist.all_gather_object(out, obj, group=group)
            return out

        node = node if node is not None and node >= 0 else -1
        # every decision below is taken from the same gathered values on every rank
        ranks = gather((local_rank, node, node_mem_free(node), mem_available()))
        avail = ranks[[r[0] for r in ranks].index(0)][3] if any(r[0] == 0 for r in ranks) \
            else ranks[0][3]
        nodes = sorted({r[1] for r in ranks})
        split = per_node and len(nodes) > 1 and -1 not in nodes
        if split:
            fits = all(free >= nbytes + self._NODE_HEADROOM for _, _, free, _ in ranks)
            split = fits and (not avail or avail >= len(nodes) * nbytes + headroom)
        key_of = {lr: (n if split else 0) for lr, n, _, _ in ranks}
        owner_of = {}
        for lr in sorted(key_of):
            owner_of.setdefault(key_of[lr], lr)
        self.copies = len(owner_of)
        self.rank_nodes = {lr: n for lr, n, _, _ in ranks}
        self.owner = owner_of[key_of[local_rank]] == local_rank
        # the node this rank's copy is placed on (None: default placement)
        self.node = node if (split or (len(nodes) == 1 and node >= 0)) else None
        err = None
        info = None
        if self.owner:
            if not split and avail and nbytes + headroom > avail:
                err = (f"shared expert store needs {nbytes / GiB:.1f} GiB + {headroom / GiB:.0f} "
                       f"GiB headroom, only {avail / GiB:.1f} GiB available")
            else:
                fd = os.memfd_create("d3_expert_store", 0)
                os.ftruncate(fd, nbytes)
                self.fd = fd
                info = (os.getpid(), fd)
        infos = gather((local_rank, err if err else info))
        errs = [x for _, x in infos if isinstance(x, str)]
        if errs:
            if self.owner and info is not None:
                os.close(self.fd)
            raise MemoryError(errs[0])
        files = {key_of[lr]: x for lr, x in infos if x is not None}
        if not self.owner:
            pid, fd = files[key_of[local_rank]]
            self.fd = os.open(f"/proc/{pid}/fd/{fd}", os.O_RDWR)
        self._primary_file = files[key_of[0]] if 0 in key_of else None
        self.mm = mmap.mmap(self.fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.buf = torch.frombuffer(self.mm, dtype=torch.uint8)
        # place the pages before anything touches them
        self.bound = (self.owner and self.node is not None
                      and bind_to_node(self.buf.data_ptr(), nbytes, self.node))
        self.chunks = []
        self.regions = []          # (offset, bytes) of every take(), registered one by one
        self.registered = False
        self._off = 0

    def copy_from_primary(self, threads: int = 16) -> None:
        """Fill this copy with local rank 0's bytes (the owner of another
        node's copy, after local rank 0 has filled its own)."""
        if self.primary or not self.owner:
            return
        pid, fd = self._primary_file
        sfd = os.open(f"/proc/{pid}/fd/{fd}", os.O_RDWR)
        try:
            smm = mmap.mmap(sfd, self.nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(sfd)
        src = torch.frombuffer(smm, dtype=torch.uint8)
        nt = torch.get_num_threads()
        torch.set_num_threads(max(nt, threads))
        try:
            for off in range(0, self.nbytes, _CHUNK):
                n = min(_CHUNK, self.nbytes - off)
                self.buf[off:off + n].copy_(src[off:off + n])
        finally:
            torch.set_num_threads(nt)
            del src
            smm.close()

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
