"""Parity of the one-process-per-GPU mode (launched by tests/test_gpu_multiprocess.py under torchrun).

Each process is one rank of a multi-process dt_comm (IPC-mapped peers, buffers in the symmetric heap, and the
NVLS buffer where the switch supports it). Every rank generates every rank's seeded inputs on the CPU, runs
the collectives on its GPU through the C ABI, and checks its output against the oracle restatement:
bit-exact for the copies and the rank-order reductions, within the north-star tolerance for NVLS.
"""

import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from dtorch_b200 import capi  # noqa: E402
from dtorch_b200.multiprocess import create_rank_comm, device_view, setup_nvls  # noqa: E402
from oracle.oracle import Restatement, shard_sizes  # noqa: E402
from tests.helpers import assert_close, raw_from_torch  # noqa: E402

R = Restatement()
OUT_OFF = 32 << 20


def main():
    rank, n = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    comm = create_rank_comm(64 << 20, local)
    base, _ = comm.heap(rank)
    stream = torch.cuda.current_stream(dev).cuda_stream
    failures = []

    def check(name, ok):
        if not ok:
            failures.append(name)

    def bufs(in_numel, out_numel, dtype, b=base):
        return device_view(b, in_numel, dtype, dev), device_view(b + OUT_OFF, out_numel, dtype, dev)

    # all-reduce: one-shot (small) and two-shot, bf16 and fp32, rank-order fp32 fold
    for dtype, code in ((torch.bfloat16, capi.DT_BFLOAT16), (torch.float32, capi.DT_FLOAT32)):
        for count in (1000, (1 << 20) + 3):
            g = torch.Generator().manual_seed(count + code)
            parts = [torch.randn(count, generator=g).to(dtype) for _ in range(n)]
            x, y = bufs(count, count, dtype)
            x.copy_(parts[rank].to(dev))
            comm.all_reduce(rank, x.data_ptr(), y.data_ptr(), count, code, 0, stream)
            torch.cuda.synchronize()
            want = R.fold_sum([raw_from_torch(p) for p in parts], code, storage_round=False)
            check(f"all_reduce {dtype} {count}", np.array_equal(raw_from_torch(y), want))
    # reduce-scatter: aligned chunks and odd chunks (element path)
    for out_count in (4096, 4099):
        g = torch.Generator().manual_seed(out_count)
        parts = [torch.randn(n * out_count, generator=g) for _ in range(n)]
        x, y = bufs(n * out_count, out_count, torch.float32)
        x.copy_(parts[rank].to(dev))
        comm.reduce_scatter(rank, x.data_ptr(), y.data_ptr(), out_count, capi.DT_FLOAT32, 0, stream)
        torch.cuda.synchronize()
        want = R.reduce_scatter([p.numpy() for p in parts], 0, storage_round=False)[rank]
        check(f"reduce_scatter {out_count}", np.array_equal(y.cpu().numpy(), want))
    # all-gather along dim 1, uneven shards
    full_shape = (6, 5 * n + 3, 4)
    lens = shard_sizes(full_shape[1], n)
    g = torch.Generator().manual_seed(11)
    shards = [torch.randn(6, lens[r], 4, generator=g).to(torch.bfloat16) for r in range(n)]
    x, y = bufs(shards[rank].numel(), 6 * sum(lens) * 4, torch.bfloat16)
    x.copy_(shards[rank].reshape(-1).to(dev))
    comm.all_gather(rank, x.data_ptr(), y.data_ptr(), 6, lens, 4 * 2, stream)
    torch.cuda.synchronize()
    want = R.all_gather([raw_from_torch(s) for s in shards], 1)
    check("all_gather dim1 uneven", np.array_equal(raw_from_torch(y).reshape(want.shape), want))
    # all-to-all Shard(1) -> Shard(2), uneven both ways
    S, H, D = 7 * n + 3, 2 * n + 1, 8
    src_lens = shard_sizes(S, n)
    g = torch.Generator().manual_seed(12)
    parts = [torch.randn(1, src_lens[r], H, D, generator=g).to(torch.bfloat16) for r in range(n)]
    split = shard_sizes(H, n)
    x, y = bufs(parts[rank].numel(), S * split[rank] * D, torch.bfloat16)
    x.copy_(parts[rank].reshape(-1).to(dev))
    comm.all_to_all(rank, x.data_ptr(), y.data_ptr(), [1, src_lens[rank], H, D], 1, 2, src_lens, 2, stream)
    torch.cuda.synchronize()
    want = R.all_to_all([raw_from_torch(p) for p in parts], 1, 2)[rank]
    check("all_to_all S1->S2 uneven", np.array_equal(raw_from_torch(y).reshape(want.shape), want))
    # NVLS all-reduce across processes (multicast handle handed over as a file descriptor)
    nvls = setup_nvls(comm, 64 << 20)
    if nvls:
        nb, _ = comm.nvls_buffer(rank)
        for dtype, code, name in ((torch.bfloat16, capi.DT_BFLOAT16, "bfloat16"), (torch.float32, capi.DT_FLOAT32, "float32")):
            count = (1 << 20) + 64
            g = torch.Generator().manual_seed(21 + code)
            parts = [torch.randn(count, generator=g).to(dtype) for _ in range(n)]
            x, y = bufs(count, count, dtype, nb)
            x.copy_(parts[rank].to(dev))
            comm.all_reduce(rank, x.data_ptr(), y.data_ptr(), count, code, capi.DT_ALGO_NVLS, stream)
            torch.cuda.synchronize()
            want = R.fold_sum([raw_from_torch(p) for p in parts], code, storage_round=False)
            try:
                assert_close(raw_from_torch(y), want, name)
            except AssertionError:
                failures.append(f"nvls all_reduce {name}")
    check("device error word", comm.error(rank) == capi.DT_OK)
    bad = torch.tensor([len(failures)], device=dev)
    dist.all_reduce(bad)
    if failures:
        print(f"rank {rank} failures: {failures}", flush=True)
    dist.barrier()
    comm.destroy()
    dist.destroy_process_group()
    if int(bad.item()) == 0 and rank == 0:
        print(f"MP PARITY OK n={n} nvls={nvls}", flush=True)
    sys.exit(0 if int(bad.item()) == 0 else 1)


if __name__ == "__main__":
    main()
