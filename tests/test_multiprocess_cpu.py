"""CPU, world size 2 over gloo: the host side of the one-process-per-GPU mode (dtorch_b200/multiprocess.py) --
the handle exchange, the file-descriptor handoff and the NVLS set-up order -- with a stand-in communicator, so
no GPU is touched."""

import os
import socket
import tempfile

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from dtorch_b200 import multiprocess


class FakeComm:
    """Records what the set-up calls do; its 'NVLS buffer' is a temporary file shared by descriptor."""

    def __init__(self, rank, nvls=True):
        self.rank = rank
        self.nvls = nvls
        self.imported = None
        self.calls = []

    def export_handle(self):
        return bytes([self.rank]) * 8

    def import_handles(self, handles):
        self.imported = handles

    def nvls_supported(self):
        return self.nvls

    def nvls_create(self, nbytes):
        self.calls.append("create")
        f = tempfile.TemporaryFile()
        f.write(b"nvls-object")
        f.flush()
        self._file = f
        return os.dup(f.fileno())

    def nvls_attach(self, fd, nbytes):
        self.calls.append("attach")
        self.attached = os.pread(fd, 11, 0)

    def nvls_bind(self):
        self.calls.append("bind")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = FakeComm(rank)
        multiprocess.exchange_handles(comm)
        ok = multiprocess.setup_nvls(comm, 1 << 20)
        mixed = FakeComm(rank, nvls=(rank == 0))  # one rank without multicast: nothing is set up anywhere
        ok_mixed = multiprocess.setup_nvls(mixed, 1 << 20)
        q.put((rank, comm.imported, ok, comm.calls, getattr(comm, "attached", None), ok_mixed, mixed.calls))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_fd_handoff_and_nvls_order():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        _, imported, ok, calls, attached, ok_mixed, mixed_calls = res[rank]
        assert imported == [bytes([r]) * 8 for r in range(world)]
        assert ok is True
        assert calls == (["create", "attach", "bind"] if rank == 0 else ["attach", "bind"])
        assert attached == b"nvls-object"  # the descriptor rank 0 created, received over the socket
        assert ok_mixed is False and mixed_calls == []
