"""GPU parity of the same-device kernels (all ranks' buffers on cuda:0, one launch) through the C ABI,
against the reference's own outputs (golden fixtures) and the oracle restatement."""

import numpy as np
import pytest
import torch

from dtorch_b200 import capi
from oracle.oracle import Restatement, shard_sizes
from tests.gpu_util import launches, np_raw, to_dev
from tests.helpers import DT_CODE, assert_close, golden_cases, raw_from_torch

pytestmark = pytest.mark.gpu
R = Restatement()
TD = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("case", golden_cases("all_reduce"), ids=lambda c: c[0])
def test_local_all_reduce_golden(case):
    name, meta, ins, outs = case
    dt = meta["dtype"]
    code = DT_CODE[dt]
    d_in = [to_dev(a, dt, 0) for a in ins]
    out = torch.empty_like(d_in[0])
    n0 = launches()
    # reference rounding: bit-exact against the reference's fold
    capi.local_all_reduce([t.data_ptr() for t in d_in], out.data_ptr(), out.numel(), code, capi.DT_ACCUM_STORAGE)
    torch.cuda.synchronize()
    assert launches() > n0
    assert np.array_equal(np_raw(out), outs[0]), name
    # default fp32 accumulation: bit-exact against the restatement in that mode, within tolerance of the reference
    capi.local_all_reduce([t.data_ptr() for t in d_in], out.data_ptr(), out.numel(), code, capi.DT_ACCUM_FP32)
    torch.cuda.synchronize()
    assert np.array_equal(np_raw(out), R.fold_sum(ins, code, storage_round=False))
    assert_close(np_raw(out), outs[0], dt)


@pytest.mark.parametrize("case", golden_cases("reduce_scatter"), ids=lambda c: c[0])
def test_local_reduce_scatter_golden(case):
    name, meta, ins, outs = case
    dt = meta["dtype"]
    code = DT_CODE[dt]
    n = meta["n"]
    d_in = [to_dev(a, dt, 0) for a in ins]
    d_out = [torch.empty(ins[0].size // n, dtype=TD[dt], device="cuda:0") for _ in range(n)]
    capi.local_reduce_scatter([t.data_ptr() for t in d_in], [t.data_ptr() for t in d_out], d_out[0].numel(), code,
                              capi.DT_ACCUM_STORAGE)
    torch.cuda.synchronize()
    for r in range(n):
        assert np.array_equal(np_raw(d_out[r]), outs[r]), (name, r)
    capi.local_reduce_scatter([t.data_ptr() for t in d_in], [t.data_ptr() for t in d_out], d_out[0].numel(), code, 0)
    torch.cuda.synchronize()
    want = R.reduce_scatter(ins, code, storage_round=False)
    for r in range(n):
        assert np.array_equal(np_raw(d_out[r]), want[r]), (name, r)


@pytest.mark.parametrize("case", golden_cases("all_gather"), ids=lambda c: c[0])
def test_local_all_gather_golden(case):
    name, meta, ins, outs = case
    dt, dim = meta["dtype"], meta["dim"]
    d_in = [to_dev(a, dt, 0) for a in ins]
    shape = list(ins[0].shape)
    outer = int(np.prod(shape[:dim], dtype=np.int64))
    inner = int(np.prod(shape[dim + 1:], dtype=np.int64)) * ins[0].itemsize
    lens = [a.shape[dim] for a in ins]
    out = torch.empty(outs[0].size, dtype=TD[dt], device="cuda:0")
    capi.local_all_gather([t.data_ptr() for t in d_in], out.data_ptr(), outer, lens, inner)
    torch.cuda.synchronize()
    assert np.array_equal(np_raw(out).reshape(outs[0].shape), outs[0]), name


@pytest.mark.parametrize("case", golden_cases("all_to_all"), ids=lambda c: c[0])
def test_local_all_to_all_golden(case):
    name, meta, ins, outs = case
    dt, sd, dd = meta["dtype"], meta["src_dim"], meta["dst_dim"]
    n = meta["n"]
    d_in = [to_dev(a, dt, 0) for a in ins]
    d_out = [torch.empty(o.size, dtype=TD[dt], device="cuda:0") for o in outs]
    capi.local_all_to_all([t.data_ptr() for t in d_in], [t.data_ptr() for t in d_out], list(ins[0].shape), sd, dd,
                          [a.shape[sd] for a in ins], ins[0].itemsize)
    torch.cuda.synchronize()
    for r in range(n):
        assert np.array_equal(np_raw(d_out[r]).reshape(outs[r].shape), outs[r]), (name, r)


@pytest.mark.parametrize("dt", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("n", [2, 3, 8])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_local_all_reduce_large_and_misaligned(dt, n, offset):
    # sizes that are not multiples of the vector width and buffers that start off a 16-byte boundary
    count = (1 << 20) + 5
    g = torch.Generator().manual_seed(11 + n + offset)
    host = [torch.randn(count + offset, generator=g).to(TD[dt]) for _ in range(n)]
    d_in = [h.to("cuda:0")[offset:] for h in host]
    out_full = torch.empty(count + offset, dtype=TD[dt], device="cuda:0")
    out = out_full[offset:]
    capi.local_all_reduce([t.data_ptr() for t in d_in], out.data_ptr(), count, DT_CODE[dt], 0)
    torch.cuda.synchronize()
    want = R.fold_sum([raw_from_torch(h[offset:]) for h in host], DT_CODE[dt], storage_round=False)
    assert np.array_equal(np_raw(out), want)


def test_local_all_to_all_ulysses_shape():
    # Ulysses swap Shard(1) -> Shard(2) on (1, S, H, D) at a reduced size, n = 8, uneven heads
    n, S, H, Dh = 8, 1024, 20, 64
    g = torch.Generator().manual_seed(5)
    lens = shard_sizes(S, n)
    host = [torch.randn(1, l, H, Dh, generator=g).to(torch.bfloat16) for l in lens]
    d_in = [h.to("cuda:0") for h in host]
    split = shard_sizes(H, n)
    d_out = [torch.empty(1, S, split[k], Dh, dtype=torch.bfloat16, device="cuda:0") for k in range(n)]
    capi.local_all_to_all([t.data_ptr() for t in d_in], [t.data_ptr() for t in d_out], [1, lens[0], H, Dh], 1, 2,
                          lens, 2)
    torch.cuda.synchronize()
    full = torch.cat(host, dim=1)
    for k in range(n):
        off = sum(split[:k])
        assert torch.equal(d_out[k].cpu(), full[:, :, off:off + split[k]])


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("count,chunk", [(1000, 0), (100_003, 4096), ((1 << 20) + 5, 64 << 10)])
def test_local_all_reduce_from_host_buffers(dt, count, chunk):
    """dt_local_all_reduce_host: pinned host partials in, pinned host sum out, one reduction per chunk; two
    back-to-back calls reuse the staging buffers in order."""
    n = 8
    code, td = DT_CODE[dt], TD[dt]
    es = torch.tensor([], dtype=td).element_size()
    g = torch.Generator().manual_seed(count)
    hosts = [[torch.randn(count, generator=g).to(td).pin_memory() for _ in range(n)] for _ in range(2)]
    dev = [torch.empty(count, dtype=td, device="cuda:0") for _ in range(n)]
    dout = torch.empty(count, dtype=td, device="cuda:0")
    houts = [torch.empty(count, dtype=td).pin_memory() for _ in range(2)]
    s = torch.cuda.Stream(device=0)
    n0 = launches()
    for host, hout in zip(hosts, houts):
        capi.local_all_reduce_host([h.data_ptr() for h in host], [d.data_ptr() for d in dev], dout.data_ptr(),
                                   hout.data_ptr(), count, code, 0, chunk, s.cuda_stream)
    s.synchronize()
    chunk_elems = max(16, (chunk or (16 << 20)) // 16 * 16) // es
    assert launches() - n0 == 2 * ((count + chunk_elems - 1) // chunk_elems)
    for host, hout in zip(hosts, houts):
        want = R.fold_sum([raw_from_torch(h) for h in host], code, storage_round=False)
        assert np.array_equal(raw_from_torch(hout), want)
    # reference rounding on request, as dt_local_all_reduce
    capi.local_all_reduce_host([h.data_ptr() for h in hosts[0]], [d.data_ptr() for d in dev], dout.data_ptr(),
                               houts[0].data_ptr(), count, code, capi.DT_ACCUM_STORAGE, chunk, s.cuda_stream)
    s.synchronize()
    assert np.array_equal(raw_from_torch(houts[0]), R.fold_sum([raw_from_torch(h) for h in hosts[0]], code, True))


@pytest.mark.parametrize("chunk", [0, 4096])
def test_local_all_reduce_from_host_buffers_in_place(chunk):
    """dt_local_all_reduce_host with dev_out == dev_ins[2] and host_out == host_ins[1]: the sum lands in rank 1's
    host partial and matches the rank-order fold of the original partials."""
    n, count, dt = 4, 50_021, "bfloat16"
    code, td = DT_CODE[dt], TD[dt]
    g = torch.Generator().manual_seed(77)
    host = [torch.randn(count, generator=g).to(td).pin_memory() for _ in range(n)]
    want = R.fold_sum([raw_from_torch(h) for h in host], code, storage_round=False)
    dev = [torch.empty(count, dtype=td, device="cuda:0") for _ in range(n)]
    s = torch.cuda.Stream(device=0)
    capi.local_all_reduce_host([h.data_ptr() for h in host], [d.data_ptr() for d in dev], dev[2].data_ptr(),
                               host[1].data_ptr(), count, code, 0, chunk, s.cuda_stream)
    s.synchronize()
    assert np.array_equal(raw_from_torch(host[1]), want)
    assert np.array_equal(np_raw(dev[2]), want)


@pytest.mark.parametrize("dt,shape,sd,dd", [
    ("bfloat16", (4096, 64), 0, 1),        # 16-byte runs per (row, destination)
    ("float32", (2048, 24), 0, 1),         # 12-byte runs: 4-byte accesses, uneven split of 24 over 8 ranks
    ("float16", (3, 1000, 10, 2), 1, 2),   # 4-byte runs under two outer dims
])
def test_local_all_to_all_short_rows(dt, shape, sd, dd):
    """All-to-alls whose rows are far shorter than a copy item: several whole rows per warp item, one access per
    lane, bit-exact against the restatement."""
    n = 8
    g = torch.Generator().manual_seed(sum(shape))
    lens = shard_sizes(shape[sd], n)
    host = []
    for l in lens:
        s = list(shape)
        s[sd] = l
        host.append(torch.randn(*s, generator=g).to(TD[dt]))
    split = shard_sizes(shape[dd], n)
    d_in = [h.to("cuda:0") for h in host]
    d_out = []
    for k in range(n):
        s = list(shape)
        s[dd] = split[k]
        d_out.append(torch.empty(*s, dtype=TD[dt], device="cuda:0"))
    in_shape = list(host[0].shape)
    capi.local_all_to_all([t.data_ptr() for t in d_in], [t.data_ptr() for t in d_out], in_shape, sd, dd, lens,
                          host[0].element_size())
    torch.cuda.synchronize()
    want = R.all_to_all([raw_from_torch(h) for h in host], sd, dd)
    for k in range(n):
        assert np.array_equal(np_raw(d_out[k]).reshape(want[k].shape), want[k]), k
