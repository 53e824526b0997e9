"""One process per GPU: building a dt_comm over an initialised torch.distributed process group.

DTorch itself keeps every rank in one process (``capi.Comm(devices)``); launchers such as torchrun start one
process per GPU instead. Then each process holds one rank of a multi-process communicator whose peers are
reached through IPC-mapped slabs, and every buffer a collective touches on a peer lives in the communicator's
symmetric heap (or its NVLS buffer).
"""

from __future__ import annotations

import contextlib
import os
import socket
import tempfile

import torch
import torch.distributed as dist

from . import capi


def exchange_handles(comm) -> None:
    """Give every rank every rank's exported communicator handle, in rank order, and import them."""
    handles = [None] * dist.get_world_size()
    dist.all_gather_object(handles, comm.export_handle())
    comm.import_handles(handles)


def create_rank_comm(heap_bytes: int, local_device: int) -> capi.Comm:
    """This process's rank of a communicator spanning the default process group, peers mapped."""
    rank, n = dist.get_rank(), dist.get_world_size()
    comm = capi.Comm.for_rank(n, rank, local_device, heap_bytes)
    exchange_handles(comm)
    return comm


def share_fd(fd: int, tag: str) -> int:
    """Hand rank 0's file descriptor to every other rank (SCM_RIGHTS over a Unix socket); returns this rank's
    descriptor (rank 0's own, or the received duplicate, which the caller closes)."""
    rank, n = dist.get_rank(), dist.get_world_size()
    path = os.path.join(tempfile.gettempdir(), f"dtb_{os.getuid()}_{os.environ.get('MASTER_PORT', '0')}_{tag}.sock")
    if rank == 0:
        if os.path.exists(path):
            os.unlink(path)
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        srv.bind(path)
        srv.listen(n)
        dist.barrier()
        for _ in range(n - 1):
            conn, _ = srv.accept()
            socket.send_fds(conn, [b"f"], [fd])
            conn.close()
        srv.close()
        os.unlink(path)
        dist.barrier()
        return fd
    dist.barrier()
    c = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    c.connect(path)
    _, fds, _, _ = socket.recv_fds(c, 16, 1)
    c.close()
    dist.barrier()
    return fds[0]


def setup_nvls(comm: capi.Comm, nbytes: int) -> bool:
    """Bind an NVLS buffer of `nbytes` on every rank (create -> hand the fd over -> attach -> barrier -> bind).
    Returns False, with nothing allocated, when any rank's device lacks NVLink multicast."""
    ok = torch.tensor([1 if comm.nvls_supported() else 0], device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok.item()) == 0:
        return False
    fd = comm.nvls_create(nbytes) if dist.get_rank() == 0 else -1
    fd = share_fd(fd, "nvls")
    comm.nvls_attach(fd, nbytes)
    dist.barrier()  # every device added before any rank binds memory
    comm.nvls_bind()
    dist.barrier()
    os.close(fd)
    return True


class _CAI:
    def __init__(self, ptr, numel, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (numel,), "typestr": typestr, "version": 3,
                                         "strides": None}


def device_view(ptr: int, numel: int, dtype, device) -> torch.Tensor:
    """A 1-D torch view of `numel` elements of device memory at `ptr` (a heap or NVLS buffer)."""
    ts = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.float16: "<i2", torch.uint8: "|u1"}[dtype]
    t = torch.as_tensor(_CAI(ptr, numel, ts), device=device)
    return t.view(dtype) if dtype in (torch.bfloat16, torch.float16) else t


def parse_cpulist(text: str) -> set:
    """CPUs of a Linux cpulist ("0-55,112-167")."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def device_local_cpus(device: int) -> set:
    """CPUs on the NUMA node the GPU's PCIe link attaches to (sysfs ``local_cpulist``); empty if unknown."""
    p = torch.cuda.get_device_properties(device)
    path = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist"
    try:
        with open(path) as f:
            return parse_cpulist(f.read())
    except OSError:
        return set()


@contextlib.contextmanager
def near_device(device: int, cpus=None):
    """Run the block on the calling thread with its CPUs limited to those local to `device`, so host memory
    allocated in the block -- pinned staging buffers above all -- lands on the GPU's own NUMA node (the kernel's
    default local placement) and their DMA does not cross the socket interconnect when every GPU of the box
    copies at once. The thread's previous CPU set is restored afterwards; where the local CPUs are unknown or
    not allowed to this process, the block runs unchanged. Yields the CPU set used (None when unchanged)."""
    local = set(cpus) if cpus is not None else device_local_cpus(device)
    old = os.sched_getaffinity(0)
    use = local & old
    if not use or use == old:
        yield None
        return
    os.sched_setaffinity(0, use)
    try:
        yield use
    finally:
        os.sched_setaffinity(0, old)
