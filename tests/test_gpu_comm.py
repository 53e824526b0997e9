"""GPU parity of the communicator entry points, called the way the reference calls its ThreadGroup: one host
thread per rank, each on its own stream (dtorch/tests/test_nccl.cc:27-65).

* same-device communicator: every rank on cuda:0 (the reference's ThreadGroupSameDeviceBackend mode)
* peer communicator: rank r on cuda:r, kernels moving data through peer HBM (needs >= 2 GPUs)
* bounded waits: a peer that never arrives ends in DT_ERR_TIMEOUT, not a hang
"""

import ctypes

import numpy as np
import pytest
import torch

from dtorch_b200 import capi
from oracle.oracle import Restatement, shard_sizes
from tests.gpu_util import np_raw, run_ranks, to_dev, view_device_memory
from tests.helpers import DT_CODE, assert_close, golden_cases, raw_from_torch

pytestmark = pytest.mark.gpu
R = Restatement()
TD = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture(autouse=True)
def _need_gpu():
    if ngpu() < 1:
        pytest.skip("no CUDA device")


def devices_for(n, mode):
    if mode == "same":
        return [0] * n
    if ngpu() < n:
        pytest.skip(f"peer mode with {n} ranks needs {n} GPUs")
    return list(range(n))


def run_case(comm, devs, meta, ins, flags=0):
    """Run one golden case through the communicator; returns per-rank raw outputs."""
    n = meta["n"]
    dt = meta["dtype"]
    op = meta["op"]
    code = DT_CODE[dt]
    d_in = [to_dev(a, dt, devs[r]) for r, a in enumerate(ins)]
    streams = [torch.cuda.Stream(device=devs[r]) for r in range(n)]
    outs = [None] * n

    def rank_fn(r):
        with torch.cuda.device(devs[r]):
            s = streams[r]
            s.wait_stream(torch.cuda.current_stream(devs[r]))
            with torch.cuda.stream(s):
                x = d_in[r]
                if op == "all_reduce":
                    o = torch.empty_like(x)
                    comm.all_reduce(r, x.data_ptr(), o.data_ptr(), x.numel(), code, flags, s.cuda_stream)
                elif op == "reduce_scatter":
                    o = torch.empty(x.numel() // n, dtype=x.dtype, device=x.device)
                    comm.reduce_scatter(r, x.data_ptr(), o.data_ptr(), o.numel(), code, flags, s.cuda_stream)
                elif op == "all_gather":
                    dim = meta["dim"]
                    shp = list(ins[r].shape)
                    lens = [a.shape[dim] for a in ins]
                    outer = int(np.prod(shp[:dim], dtype=np.int64))
                    inner = int(np.prod(shp[dim + 1:], dtype=np.int64)) * ins[r].itemsize
                    o = torch.empty(outer * sum(lens) * inner // ins[r].itemsize, dtype=x.dtype, device=x.device)
                    comm.all_gather(r, x.data_ptr(), o.data_ptr(), outer, lens, inner, s.cuda_stream)
                else:
                    sd, dd = meta["src_dim"], meta["dst_dim"]
                    lens = [a.shape[sd] for a in ins]
                    split = shard_sizes(ins[0].shape[dd], n)
                    numel = ins[r].size // ins[r].shape[sd] * sum(lens) // ins[r].shape[dd] * split[r]
                    o = torch.empty(numel, dtype=x.dtype, device=x.device)
                    comm.all_to_all(r, x.data_ptr(), o.data_ptr(), list(ins[r].shape), sd, dd, lens,
                                    ins[r].itemsize, s.cuda_stream)
                outs[r] = o
            s.synchronize()

    run_ranks(n, rank_fn)
    return [np_raw(o) for o in outs]


@pytest.mark.parametrize("mode", ["same", "peer"])
@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c[0])
def test_comm_golden(case, mode):
    name, meta, ins, outs = case
    n, op, dt = meta["n"], meta["op"], meta["dtype"]
    devs = devices_for(n, mode)
    comm = capi.Comm(devs)
    try:
        comm.set_timeout_ms(20000)
        reduce_op = op in ("all_reduce", "reduce_scatter")
        got = run_case(comm, devs, meta, ins, flags=capi.DT_ACCUM_STORAGE if reduce_op else 0)
        for r in range(n):
            assert np.array_equal(got[r].reshape(outs[r].shape), outs[r]), (name, r)
        if reduce_op:
            # default fp32 accumulation: bit-exact vs the restatement in that mode, within tolerance of the reference
            got = run_case(comm, devs, meta, ins, flags=0)
            want = (R.fold_sum(ins, DT_CODE[dt], False) if op == "all_reduce"
                    else R.reduce_scatter(ins, DT_CODE[dt], False))
            for r in range(n):
                w = want if op == "all_reduce" else want[r]
                assert np.array_equal(got[r], w.reshape(-1)), (name, r)
                assert_close(got[r], outs[r].reshape(-1), dt)
        assert comm.error(0) == capi.DT_OK
    finally:
        comm.destroy()


def _random_case(rng, n):
    """One seeded random collective (op, dtype, shape, dims, uneven shards) with the restatement's answer."""
    op = str(rng.choice(["all_reduce", "reduce_scatter", "all_gather", "all_to_all"]))
    dt = str(rng.choice(["float32", "bfloat16", "float16"]))
    td = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dt]
    g = torch.Generator().manual_seed(int(rng.integers(1 << 30)))

    def tensor(shape):
        return raw_from_torch(torch.randn(*shape, generator=g).to(td))

    meta = {"n": n, "op": op, "dtype": dt}
    if op in ("all_reduce", "reduce_scatter"):
        count = int(rng.integers(1, 3000)) * (n if op == "reduce_scatter" else 1)
        ins = [tensor([count]) for _ in range(n)]
        want = ([R.fold_sum(ins, DT_CODE[dt], False)] * n if op == "all_reduce"
                else R.reduce_scatter(ins, DT_CODE[dt], False))
        return meta, ins, want
    ndim = int(rng.integers(1 if op == "all_gather" else 2, 5))
    shape = [int(rng.integers(1, 9)) for _ in range(ndim)]
    dim = int(rng.integers(ndim))
    lens = shard_sizes(int(rng.integers(n, 4 * n + 3)), n)
    if op == "all_gather":
        ins = []
        for l in lens:
            s = list(shape)
            s[dim] = l
            ins.append(tensor(s))
        meta["dim"] = dim
        return meta, ins, [R.all_gather(ins, dim)] * n
    dd = int(rng.choice([d for d in range(ndim) if d != dim]))
    shape[dd] = max(shape[dd], n) + int(rng.integers(0, 3))
    ins = []
    for l in lens:
        s = list(shape)
        s[dim] = l
        ins.append(tensor(s))
    meta["src_dim"], meta["dst_dim"] = dim, dd
    return meta, ins, R.all_to_all(ins, dim, dd)


@pytest.mark.parametrize("mode", ["same", "peer"])
@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_comm_random_cases_match_restatement(mode, n):
    """Seeded random collectives (ops, dtypes, ranks of 1-4 dims, every dim pair, uneven shards, odd sizes)
    through the C ABI: gathers and all-to-alls bit-exact, reductions bit-exact against the fp32-accumulate
    restatement."""
    devs = devices_for(n, mode)
    rng = np.random.default_rng(1000 + n)
    comm = capi.Comm(devs)
    try:
        comm.set_timeout_ms(20000)
        for i in range(24):
            meta, ins, want = _random_case(rng, n)
            got = run_case(comm, devs, meta, ins, flags=0)
            for r in range(n):
                assert np.array_equal(got[r], np.asarray(want[r]).reshape(-1)), (i, meta, r)
        assert comm.error(0) == capi.DT_OK
    finally:
        comm.destroy()


@pytest.mark.parametrize("algo", [capi.DT_ALGO_ONESHOT, capi.DT_ALGO_TWOSHOT])
@pytest.mark.parametrize("count", [1, 7, 4096 + 3, (1 << 21) + 9])
def test_peer_all_reduce_algorithms(algo, count):
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    devs = list(range(n))
    comm = capi.Comm(devs)
    try:
        g = torch.Generator().manual_seed(count)
        host = [torch.randn(count, generator=g).to(torch.bfloat16) for _ in range(n)]
        d_in = [h.to(f"cuda:{r}") for r, h in enumerate(host)]
        outs = [torch.empty_like(t) for t in d_in]

        def fn(r):
            with torch.cuda.device(r):
                comm.all_reduce(r, d_in[r].data_ptr(), outs[r].data_ptr(), count, capi.DT_BFLOAT16, algo,
                                torch.cuda.current_stream(r).cuda_stream)
                torch.cuda.current_stream(r).synchronize()

        for _ in range(3):  # back-to-back calls reuse the flags with growing epochs
            run_ranks(n, fn)
        want = R.fold_sum([raw_from_torch(h) for h in host], 1, storage_round=False)
        for r in range(n):
            assert np.array_equal(np_raw(outs[r]), want), r
    finally:
        comm.destroy()


def test_peer_in_place_all_reduce_and_heap_buffers():
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    devs = list(range(n))
    count = (1 << 20) + 16
    comm = capi.Comm(devs, heap_bytes=8 << 20)
    try:
        g = torch.Generator().manual_seed(1)
        host = [torch.randn(count, generator=g) for _ in range(n)]
        bufs = []
        for r in range(n):
            base, size = comm.heap(r)
            assert size == 8 << 20
            t = view_device_memory(base, count, torch.float32, r)
            t.copy_(host[r].to(f"cuda:{r}"))
            bufs.append(t)
        torch.cuda.synchronize()

        def fn(r):
            with torch.cuda.device(r):
                # heap buffers: peers are reached by symmetric offset, no host rendezvous; in place
                comm.all_reduce(r, bufs[r].data_ptr(), bufs[r].data_ptr(), count, capi.DT_FLOAT32, 0,
                                torch.cuda.current_stream(r).cuda_stream)
                torch.cuda.current_stream(r).synchronize()

        run_ranks(n, fn)
        want = R.fold_sum([h.numpy() for h in host], 0, storage_round=False)
        for r in range(n):
            assert np.array_equal(bufs[r].cpu().numpy(), want)
    finally:
        comm.destroy()


@pytest.mark.parametrize("count", [1000, 64 * 1024 + 3])
def test_peer_all_reduce_some_ranks_in_place(count):
    """Even ranks reduce in place, odd ranks into a separate output: every rank still takes the same kernel
    (the algorithm is chosen from all ranks' pointers), and all get the rank-order sum."""
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    comm = capi.Comm(list(range(n)))
    try:
        g = torch.Generator().manual_seed(count)
        host = [torch.randn(count, generator=g) for _ in range(n)]
        xs = [host[r].to(f"cuda:{r}") for r in range(n)]
        ys = [xs[r] if r % 2 == 0 else torch.empty_like(xs[r]) for r in range(n)]
        torch.cuda.synchronize()

        def fn(r):
            with torch.cuda.device(r):
                s = torch.cuda.current_stream(r)
                comm.all_reduce(r, xs[r].data_ptr(), ys[r].data_ptr(), count, capi.DT_FLOAT32, 0, s.cuda_stream)
                s.synchronize()

        run_ranks(n, fn)
        want = R.fold_sum([h.numpy() for h in host], 0, storage_round=False)
        for r in range(n):
            assert np.array_equal(ys[r].cpu().numpy(), want), r
        for r in range(1, n, 2):
            assert torch.equal(xs[r].cpu(), host[r])  # out-of-place ranks keep their input
        assert comm.error(0) == capi.DT_OK
    finally:
        comm.destroy()


def test_peer_device_wait_times_out_cleanly():
    """Rank 1 never launches: rank 0's barrier kernel gives up after the 1 s limit, records DT_ERR_TIMEOUT
    in the host-mapped error word and returns; the context stays usable."""
    if ngpu() < 2:
        pytest.skip("needs >= 2 GPUs")
    comm = capi.Comm([0, 1])
    try:
        comm.set_timeout_ms(1000)
        with torch.cuda.device(0):
            s = torch.cuda.current_stream(0)
            comm.barrier(0, s.cuda_stream)
            s.synchronize()
        assert comm.error(0) == capi.DT_ERR_TIMEOUT
        x = torch.ones(16, device="cuda:0") * 2
        assert float(x.sum()) == 32.0  # the GPU still answers
    finally:
        comm.destroy()


def test_same_device_rendezvous_times_out_cleanly():
    """One rank thread never arrives: the others get DT_ERR_TIMEOUT from the host rendezvous; no kernel waits."""
    comm = capi.Comm([0, 0, 0])
    try:
        comm.set_timeout_ms(300)
        x = torch.ones(64, device="cuda:0")
        o = torch.empty_like(x)
        errs = []

        def fn(r):
            if r == 2:
                return
            try:
                comm.all_reduce(r, x.data_ptr(), o.data_ptr(), 64, capi.DT_FLOAT32, 0, 0)
            except capi.DtError as e:
                errs.append(e.status)

        run_ranks(3, fn)
        assert sorted(errs) == [capi.DT_ERR_TIMEOUT, capi.DT_ERR_TIMEOUT]
        with pytest.raises(capi.DtError) as ei:
            comm.all_reduce(0, x.data_ptr(), o.data_ptr(), 64, capi.DT_FLOAT32, 0, 0)
        assert ei.value.status == capi.DT_ERR_STATE  # broken communicator refuses further calls
    finally:
        comm.destroy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_nvls_all_reduce(dtype):
    """NVLS all-reduce (reduction inside the NVSwitch): within the north-star tolerance of the rank-order
    fold, identical on every rank and from run to run; in place. The default algorithm on NVLS buffers is the
    rank-order kernel below the switch-over size (16 MiB at 4-5 ranks, 8 MiB at 6+) and NVLS from there."""
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    devs = list(range(n))
    comm = capi.Comm(devs)
    try:
        if not comm.nvls_supported():
            pytest.skip("NVLink multicast not supported here")
        es = torch.tensor([], dtype=dtype).element_size()
        count = (1 << 20) + 64 // es  # multiple of 16 bytes, not of a power of two
        comm.nvls_alloc(2 * count * es + (1 << 20))
        code = capi.dtype_code(dtype)
        name = {torch.bfloat16: "bfloat16", torch.float32: "float32"}[dtype]
        g = torch.Generator().manual_seed(7)
        host = [torch.randn(count, generator=g).to(dtype) for _ in range(n)]
        xs, ys = [], []
        for r in range(n):
            base, size = comm.nvls_buffer(r)
            assert size >= 2 * count * es
            x = view_device_memory(base, count, dtype, r)
            y = view_device_memory(base + count * es + 4096, count, dtype, r)
            x.copy_(host[r].to(f"cuda:{r}"))
            xs.append(x)
            ys.append(y)
        torch.cuda.synchronize()
        want = R.fold_sum([raw_from_torch(h) for h in host], DT_CODE[name], storage_round=False)

        def run(flags, in_place=False):
            def fn(r):
                with torch.cuda.device(r):
                    s = torch.cuda.current_stream(r)
                    dst = xs[r] if in_place else ys[r]
                    comm.all_reduce(r, xs[r].data_ptr(), dst.data_ptr(), count, code, flags, s.cuda_stream)
                    s.synchronize()
            run_ranks(n, fn)

        run(capi.DT_ALGO_NVLS)
        first = [np_raw(y) for y in ys]
        run(capi.DT_ALGO_NVLS)
        for r in range(n):
            assert np.array_equal(np_raw(ys[r]), first[r]), "run-to-run"
            assert np.array_equal(first[r], first[0]), "ranks disagree"
            assert_close(first[r], want, name)
        assert comm.error(0) == capi.DT_OK
        for y in ys:  # default algorithm on NVLS buffers below the switch-over size: the rank-order fold
            y.zero_()
        torch.cuda.synchronize()
        run(0)
        for r in range(n):
            assert np.array_equal(np_raw(ys[r]), want)
        run(capi.DT_ALGO_NVLS, in_place=True)
        for r in range(n):
            assert np.array_equal(np_raw(xs[r]), first[0])
        with pytest.raises(capi.DtError):  # storage rounding is not available in the switch
            comm.all_reduce(0, xs[0].data_ptr(), ys[0].data_ptr(), count, code,
                            capi.DT_ALGO_NVLS | capi.DT_ACCUM_STORAGE, 0)
        with pytest.raises(capi.DtError) as e:  # nor the rank-order fold
            comm.all_reduce(0, xs[0].data_ptr(), ys[0].data_ptr(), count, code,
                            capi.DT_ALGO_NVLS | capi.DT_RANK_ORDER, 0)
        assert e.value.status == capi.DT_ERR_UNSUPPORTED
    finally:
        comm.destroy()


def test_nvls_picked_by_default_from_switch_over_size():
    """At >= 6 ranks an all-reduce on NVLS-buffer operands of 8 MiB or more reduces in the switch by default; at
    4 ranks it keeps the rank-order kernel (measured level with NVLS there)."""
    n = min(ngpu(), 8)
    if n < 4:
        pytest.skip("needs >= 4 GPUs")
    comm = capi.Comm(list(range(n)))
    try:
        if not comm.nvls_supported():
            pytest.skip("NVLink multicast not supported here")
        count = (8 << 20) // 2 + 64  # bf16, just above the switch-over size
        comm.nvls_alloc(2 * count * 2 + (1 << 20))
        g = torch.Generator().manual_seed(9)
        host = [torch.randn(count, generator=g).to(torch.bfloat16) for _ in range(n)]
        xs, ys = [], []
        for r in range(n):
            base, _ = comm.nvls_buffer(r)
            xs.append(view_device_memory(base, count, torch.bfloat16, r))
            ys.append(view_device_memory(base + count * 2 + 4096, count, torch.bfloat16, r))
            xs[r].copy_(host[r].to(f"cuda:{r}"))
        torch.cuda.synchronize()
        outs = {}
        for flags in (capi.DT_ALGO_NVLS, 0, capi.DT_RANK_ORDER):
            def fn(r):
                with torch.cuda.device(r):
                    s = torch.cuda.current_stream(r)
                    comm.all_reduce(r, xs[r].data_ptr(), ys[r].data_ptr(), count, capi.DT_BFLOAT16, flags,
                                    s.cuda_stream)
                    s.synchronize()
            run_ranks(n, fn)
            outs[flags] = [np_raw(y) for y in ys]
        want = R.fold_sum([raw_from_torch(h) for h in host], DT_CODE["bfloat16"], storage_round=False)
        for r in range(n):
            if n >= 6:
                assert np.array_equal(outs[0][r], outs[capi.DT_ALGO_NVLS][r])
            else:  # the rank-order fold, bit for bit
                assert np.array_equal(outs[0][r], want)
            assert_close(outs[0][r], want, "bfloat16")
            assert np.array_equal(outs[capi.DT_RANK_ORDER][r], want)  # pinned to the fold at any group size
    finally:
        comm.destroy()


def test_peer_collectives_replay_from_cuda_graphs():
    """Barrier epochs live in device memory, so collectives captured into a CUDA graph stay correct when the
    graph is replayed: each rank thread captures an all-reduce and an all-to-all, then replays them with new
    inputs, with eager calls in between."""
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    devs = list(range(n))
    comm = capi.Comm(devs)
    count = (1 << 20) + 8
    S, H, D = 16 * n, 2 * n, 32
    lens = shard_sizes(S, n)
    try:
        x = [torch.zeros(count, dtype=torch.bfloat16, device=f"cuda:{r}") for r in devs]
        y = [torch.zeros_like(t) for t in x]
        a_in = [torch.zeros(1, lens[r], H, D, dtype=torch.bfloat16, device=f"cuda:{r}") for r in devs]
        a_out = [torch.zeros(1, S, H // n, D, dtype=torch.bfloat16, device=f"cuda:{r}") for r in devs]
        streams = [torch.cuda.Stream(device=r) for r in devs]
        graphs = [torch.cuda.CUDAGraph() for _ in devs]

        def step(r):
            s = streams[r].cuda_stream
            comm.all_reduce(r, x[r].data_ptr(), y[r].data_ptr(), count, capi.DT_BFLOAT16, 0, s)
            comm.all_to_all(r, a_in[r].data_ptr(), a_out[r].data_ptr(), [1, lens[r], H, D], 1, 2, lens, 2, s)

        def capture(r):
            with torch.cuda.device(r):
                with torch.cuda.stream(streams[r]):
                    step(r)  # eager warm-up
                streams[r].synchronize()
                with torch.cuda.graph(graphs[r], stream=streams[r], capture_error_mode="thread_local"):
                    step(r)

        run_ranks(n, capture)
        g = torch.Generator().manual_seed(9)
        for it in range(3):
            host = [torch.randn(count, generator=g).to(torch.bfloat16) for _ in devs]
            parts = [torch.randn(1, lens[r], H, D, generator=g).to(torch.bfloat16) for r in devs]

            def replay(r):
                with torch.cuda.device(r), torch.cuda.stream(streams[r]):
                    x[r].copy_(host[r], non_blocking=False)
                    a_in[r].copy_(parts[r], non_blocking=False)
                    graphs[r].replay()
                    if it == 1:
                        step(r)  # an eager call between replays advances the same device counters
                    streams[r].synchronize()

            run_ranks(n, replay)
            want = R.fold_sum([raw_from_torch(h) for h in host], 1, storage_round=False)
            full = torch.cat(parts, dim=1)
            for r in devs:
                assert np.array_equal(np_raw(y[r]), want), (it, r)
                assert torch.equal(a_out[r].cpu(), full[:, :, r * (H // n):(r + 1) * (H // n)]), (it, r)
            assert comm.error(0) == capi.DT_OK
    finally:
        del graphs
        comm.destroy()


def _peer_or_skip(n):
    if ngpu() < n:
        pytest.skip(f"needs {n} GPUs")
    return list(range(n))


@pytest.mark.parametrize("dim", [0, 1, 2])
@pytest.mark.parametrize("inner", [4, 3, 1])  # 3 and 1 bf16 elements give odd byte runs (narrow vector paths)
def test_peer_all_gather_layouts(dim, inner):
    n = min(ngpu(), 4)
    devs = _peer_or_skip(max(n, 2))
    n = len(devs)
    full = [7, 5 * n + 3, inner]
    lens = shard_sizes(full[dim], n)
    g = torch.Generator().manual_seed(dim * 10 + inner)
    parts = []
    for r in range(n):
        shp = list(full)
        shp[dim] = lens[r]
        parts.append(torch.randn(*shp, generator=g).to(torch.bfloat16))
    comm = capi.Comm(devs)
    try:
        outs = [None] * n
        outer = int(np.prod(full[:dim]))
        inner_b = int(np.prod(full[dim + 1:])) * 2

        def fn(r):
            with torch.cuda.device(r):
                x = parts[r].to(f"cuda:{r}")
                o = torch.empty(outer * sum(lens) * inner_b // 2, dtype=torch.bfloat16, device=f"cuda:{r}")
                comm.all_gather(r, x.data_ptr(), o.data_ptr(), outer, lens, inner_b, torch.cuda.current_stream(r).cuda_stream)
                torch.cuda.current_stream(r).synchronize()
                outs[r] = o

        run_ranks(n, fn)
        want = R.all_gather([raw_from_torch(p) for p in parts], dim)
        for r in range(n):
            assert np.array_equal(np_raw(outs[r]).reshape(want.shape), want), r
    finally:
        comm.destroy()


@pytest.mark.parametrize("src_dim,dst_dim", [(1, 2), (2, 1), (0, 3), (3, 0)])
@pytest.mark.parametrize("last", [16, 3])
def test_peer_all_to_all_layouts(src_dim, dst_dim, last):
    n = min(ngpu(), 4)
    devs = _peer_or_skip(max(n, 2))
    n = len(devs)
    full = [2 * n + 1, 3 * n + 2, 2 * n + 3, last * n + 1]
    src_lens = shard_sizes(full[src_dim], n)
    g = torch.Generator().manual_seed(src_dim * 7 + dst_dim + last)
    parts = []
    for r in range(n):
        shp = list(full)
        shp[src_dim] = src_lens[r]
        parts.append(torch.randn(*shp, generator=g))
    split = shard_sizes(full[dst_dim], n)
    comm = capi.Comm(devs)
    try:
        outs = [None] * n

        def fn(r):
            with torch.cuda.device(r):
                x = parts[r].to(f"cuda:{r}")
                oshape = list(full)
                oshape[dst_dim] = split[r]
                o = torch.empty(oshape, device=f"cuda:{r}")
                comm.all_to_all(r, x.data_ptr(), o.data_ptr(), list(parts[r].shape), src_dim, dst_dim, src_lens, 4,
                                torch.cuda.current_stream(r).cuda_stream)
                torch.cuda.current_stream(r).synchronize()
                outs[r] = o

        run_ranks(n, fn)
        want = R.all_to_all([p.numpy() for p in parts], src_dim, dst_dim)
        for r in range(n):
            assert np.array_equal(outs[r].cpu().numpy(), want[r]), r
    finally:
        comm.destroy()


@pytest.mark.parametrize("out_count", [1, 13, 4096 + 5, (1 << 18) + 7])
def test_peer_reduce_scatter_fp16_odd_chunks(out_count):
    n = min(ngpu(), 8)
    devs = _peer_or_skip(max(n, 2))
    n = len(devs)
    g = torch.Generator().manual_seed(out_count)
    parts = [torch.randn(n * out_count, generator=g).to(torch.float16) for _ in range(n)]
    comm = capi.Comm(devs)
    try:
        outs = [None] * n

        def fn(r):
            with torch.cuda.device(r):
                x = parts[r].to(f"cuda:{r}")
                o = torch.empty(out_count, dtype=torch.float16, device=f"cuda:{r}")
                comm.reduce_scatter(r, x.data_ptr(), o.data_ptr(), out_count, capi.DT_FLOAT16, 0,
                                    torch.cuda.current_stream(r).cuda_stream)
                torch.cuda.current_stream(r).synchronize()
                outs[r] = o

        run_ranks(n, fn)
        want = R.reduce_scatter([raw_from_torch(p) for p in parts], 2, storage_round=False)
        for r in range(n):
            assert np.array_equal(np_raw(outs[r]), want[r]), r
    finally:
        comm.destroy()


@pytest.mark.parametrize("mode", ["same", "peer"])
@pytest.mark.parametrize("n", [2, 3, 8])
def test_list_forms_match_restatement(mode, n):
    """dt_all_to_all_list / dt_all_gather_list (c10d's list-form alltoall / allgather, one buffer per peer, uneven
    sizes, misaligned lengths): rank k's outs[i] holds exactly rank i's ins[k] (all-to-all) or rank i's input
    (all-gather), in one launch."""
    devs = devices_for(n, mode)
    rng = np.random.default_rng(77 + n)
    comm = capi.Comm(devs)
    try:
        comm.set_timeout_ms(20000)
        for it in range(4):
            sizes = rng.integers(0, 40000, size=(n, n))  # bytes rank i sends to rank k
            sizes[0, n - 1] = 1 + (it % 15)  # odd lengths force the narrow vector widths
            src = [[torch.randint(0, 255, (int(sizes[i, k]),), dtype=torch.uint8, device=f"cuda:{devs[i]}")
                    for k in range(n)] for i in range(n)]
            dst = [[torch.full((int(sizes[i, k]) + 5,), 7, dtype=torch.uint8, device=f"cuda:{devs[k]}")
                    for i in range(n)] for k in range(n)]
            gin = [torch.randint(0, 255, (int(sizes[i, 0]),), dtype=torch.uint8, device=f"cuda:{devs[i]}")
                   for i in range(n)]
            gout = [[torch.full((int(sizes[i, 0]),), 9, dtype=torch.uint8, device=f"cuda:{devs[k]}")
                     for i in range(n)] for k in range(n)]

            def fn(r):
                with torch.cuda.device(devs[r]):
                    s = torch.cuda.current_stream(devs[r]).cuda_stream
                    comm.all_to_all_list(r, [t.data_ptr() for t in src[r]], [t.numel() for t in src[r]],
                                         [t.data_ptr() for t in dst[r]], [t.numel() for t in dst[r]], s)
                    comm.all_gather_list(r, gin[r].data_ptr(), gin[r].numel(), [t.data_ptr() for t in gout[r]],
                                         [t.numel() for t in gout[r]], s)
                    torch.cuda.current_stream(devs[r]).synchronize()

            run_ranks(n, fn)
            for k in range(n):
                for i in range(n):
                    m = int(sizes[i, k])
                    got = dst[k][i].cpu()
                    assert torch.equal(got[:m], src[i][k].cpu()), (it, i, k)
                    assert torch.all(got[m:] == 7), "wrote past the sent bytes"
                    assert torch.equal(gout[k][i].cpu(), gin[i].cpu()), (it, i, k)
        assert comm.error(0) == capi.DT_OK
    finally:
        comm.destroy()


def test_list_form_rejects_oversized_sends_on_every_rank():
    n = 2
    comm = capi.Comm([0] * n)
    try:
        bufs = [torch.zeros(64, dtype=torch.uint8, device="cuda:0") for _ in range(4)]
        errs = [None] * n

        def fn(r):
            try:
                # rank 0 sends 64 bytes to rank 1, which offers room for 32
                room = [64, 64] if r == 0 else [32, 64]
                comm.all_to_all_list(r, [bufs[0].data_ptr(), bufs[1].data_ptr()], [64, 64],
                                     [bufs[2].data_ptr(), bufs[3].data_ptr()], room)
            except capi.DtError as e:
                errs[r] = e.status

        run_ranks(n, fn)
        assert errs == [capi.DT_ERR_INVALID] * n
    finally:
        comm.destroy()


@pytest.mark.parametrize("mode", ["same", "peer"])
def test_all_to_all_multi_one_launch(mode):
    """The q/k/v swap of Ulysses attention as dt_all_to_all_multi: one kernel for the three tensors (same-device
    mode included), equal to three dt_all_to_all calls, bit for bit."""
    n = 8 if mode == "same" else min(ngpu(), 8)
    if n < 2:
        pytest.skip("peer mode needs >= 2 GPUs")
    devs = devices_for(n, mode)
    S, H, D = 64, 20, 16  # (1, S, H, D) Shard(1) -> Shard(2), uneven heads at n = 8
    lens = shard_sizes(S, n)
    g = torch.Generator().manual_seed(99)
    host = [[torch.randn(1, lens[r], H, D, generator=g).to(torch.bfloat16) for r in range(n)] for _ in range(3)]
    split = shard_sizes(H, n)
    comm = capi.Comm(devs)
    try:
        comm.set_timeout_ms(20000)
        d_in = [[h.to(f"cuda:{devs[r]}") for r, h in enumerate(t)] for t in host]
        fused = [[torch.empty(1, S, split[r], D, dtype=torch.bfloat16, device=f"cuda:{devs[r]}") for r in range(n)]
                 for _ in range(3)]
        sep = [[torch.empty_like(o) for o in f] for f in fused]
        counts = {}
        import threading

        bar = threading.Barrier(n)

        def fn(r):
            with torch.cuda.device(devs[r]):
                st = torch.cuda.current_stream(devs[r])
                s = st.cuda_stream
                st.synchronize()
                bar.wait(timeout=60)
                if r == 0:
                    counts["a"] = capi.launch_count()
                bar.wait(timeout=60)
                comm.all_to_all_multi(r, [d_in[t][r].data_ptr() for t in range(3)],
                                      [fused[t][r].data_ptr() for t in range(3)], [1, lens[r], H, D], 1, 2, lens, 2, s)
                st.synchronize()
                bar.wait(timeout=60)
                if r == 0:
                    counts["b"] = capi.launch_count()
                bar.wait(timeout=60)
                for t in range(3):
                    comm.all_to_all(r, d_in[t][r].data_ptr(), sep[t][r].data_ptr(), [1, lens[r], H, D], 1, 2, lens, 2, s)
                st.synchronize()

        run_ranks(n, fn)
        for t in range(3):
            for r in range(n):
                assert torch.equal(fused[t][r].cpu(), sep[t][r].cpu()), (t, r)
            full = torch.cat(host[t], dim=1)
            for r in range(n):
                off = sum(split[:r])
                assert torch.equal(fused[t][r].cpu(), full[:, :, off:off + split[r]])
        launched = counts["b"] - counts["a"]
        # same-device: rank 0 launches the one fused kernel for the group; peer mode: one per rank
        assert launched == (1 if mode == "same" else n), launched
    finally:
        comm.destroy()
