"""GPU parity at BASELINE.json's full sizes, on one GPU: each config runs through a same-device communicator
(every rank a host thread on cuda:0, the reference's ThreadGroupSameDeviceBackend mode), and its outputs are
compared with the C restatement and, where the reference's own library was built (oracle/_ref), with the
reference's CPU thread-group path on the same seeded inputs.

  C1 all-gather  Shard(0) -> Replicate   fp32 (4096, 4096), torch.rand seed 0, 2 ranks
  C2 all-reduce  Partial -> Replicate    bf16 (8192, 8192), rank r's partial randn seed r, 8 ranks
  C3 reduce-scatter Partial -> Shard(0)  bf16 (16384, 8192), rank r's partial randn seed r, 8 ranks
  C4 all-to-all  Shard(1) -> Shard(2)    bf16 (1, 65536, 64, 128), randn seed 0, 8 ranks

These exercise the multi-CTA grid-stride paths of the kernels at 64 MiB - 2 GiB per call. Copies must be
bit-exact; reductions are bit-exact against the fp32-accumulate restatement by default and against the
reference's in-dtype fold with DT_ACCUM_STORAGE.
"""

import numpy as np
import pytest
import torch

from dtorch_b200 import capi
from oracle.oracle import Reference, Restatement, shard_sizes
from tests.gpu_util import np_raw, run_ranks
from tests.helpers import abs_sum_f64, assert_close_sum, exact_sum_f64, raw_from_torch, to_f32

pytestmark = pytest.mark.gpu
R = Restatement()


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def _gen(shape, dtype, seed, dist):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    t = torch.rand(*shape, generator=g, device="cuda:0") if dist == "rand" else \
        torch.randn(*shape, generator=g, device="cuda:0")
    return t.to(dtype)


def _same_device(n, body):
    """Run body(comm, rank, stream) on n rank threads of a same-device communicator on cuda:0."""
    comm = capi.Comm([0] * n)
    try:
        comm.set_timeout_ms(60000)
        streams = [torch.cuda.Stream(device=0) for _ in range(n)]
        for s in streams:
            s.wait_stream(torch.cuda.current_stream(0))

        def rank_fn(r):
            with torch.cuda.device(0):
                body(comm, r, streams[r])
                streams[r].synchronize()

        run_ranks(n, rank_fn)
        assert comm.error(0) == capi.DT_OK
    finally:
        comm.destroy()


def test_c1_all_gather_full_size():
    n = 2
    full = _gen((4096, 4096), torch.float32, 0, "rand")
    lens = shard_sizes(4096, n)
    shards = [t.contiguous() for t in torch.split(full, lens, 0)]
    outs = [torch.empty(4096, 4096, dtype=torch.float32, device="cuda:0") for _ in range(n)]

    def body(comm, r, s):
        comm.all_gather(r, shards[r].data_ptr(), outs[r].data_ptr(), 1, lens, 4096 * 4, s.cuda_stream)

    _same_device(n, body)
    host_shards = [raw_from_torch(t) for t in shards]
    want = R.all_gather(host_shards, 0)
    for r in range(n):
        assert np.array_equal(np_raw(outs[r]).reshape(want.shape), want), r
    if Reference.available():
        ref_outs, _ = Reference().all_gather(host_shards, 0, 0)
        for r in range(n):
            assert np.array_equal(np_raw(outs[r]).reshape(want.shape), ref_outs[r]), r


@pytest.mark.parametrize("op", ["all_reduce", "reduce_scatter"])
def test_c2_c3_reductions_full_size(op):
    n = 8
    shape = (8192, 8192) if op == "all_reduce" else (16384, 8192)
    count = shape[0] * shape[1]
    parts = [_gen(shape, torch.bfloat16, r, "randn").reshape(-1) for r in range(n)]
    out_count = count if op == "all_reduce" else count // n
    outs = [torch.empty(out_count, dtype=torch.bfloat16, device="cuda:0") for _ in range(n)]
    host = [raw_from_torch(p) for p in parts]

    def run(flags):
        def body(comm, r, s):
            if op == "all_reduce":
                comm.all_reduce(r, parts[r].data_ptr(), outs[r].data_ptr(), count, capi.DT_BFLOAT16, flags,
                                s.cuda_stream)
            else:
                comm.reduce_scatter(r, parts[r].data_ptr(), outs[r].data_ptr(), out_count, capi.DT_BFLOAT16, flags,
                                    s.cuda_stream)

        _same_device(n, body)
        return [np_raw(o) for o in outs]

    # default: fp32 accumulation in rank order, one rounding
    got = run(capi.DT_ACCUM_FP32)
    if op == "all_reduce":
        want = [R.fold_sum(host, 1, storage_round=False)] * n
    else:
        want = R.reduce_scatter(host, 1, storage_round=False)
    for r in range(n):
        assert np.array_equal(got[r], want[r]), r
    # the reference's in-dtype fold, bit for bit
    got = run(capi.DT_ACCUM_STORAGE)
    if Reference.available():
        ref = Reference()
        ref_outs, _ = ref.all_reduce(host, 1) if op == "all_reduce" else ref.reduce_scatter(host, 1)
    else:
        ref_outs = ([R.fold_sum(host, 1, storage_round=True)] * n if op == "all_reduce"
                    else R.reduce_scatter(host, 1, storage_round=True))
    for r in range(n):
        assert np.array_equal(got[r], ref_outs[r].reshape(-1)), r
    # the default mode sits within the north-star tolerance of the reference, on the scale of summation error;
    # and it is the more accurate of the two: within one bf16 rounding of the exact sum
    chunk = slice(None) if op == "all_reduce" else slice(0, out_count)
    scale = abs_sum_f64([h.reshape(-1)[chunk] for h in host], "bfloat16")
    assert_close_sum(want[0], ref_outs[0].reshape(-1), "bfloat16", scale)
    exact = exact_sum_f64([h.reshape(-1)[chunk] for h in host], "bfloat16")
    ours = to_f32(want[0].reshape(-1), "bfloat16").astype(np.float64)
    assert np.all(np.abs(ours - exact) <= 2.0 ** -8 * np.abs(exact) + 1e-6 * scale)


def test_c4_ulysses_all_to_all_full_size():
    n, gs, sd, dd = 8, (1, 65536, 64, 128), 1, 2
    full = _gen(gs, torch.bfloat16, 0, "randn")
    src_lens = shard_sizes(gs[sd], n)
    shards = [t.contiguous() for t in torch.split(full, src_lens, sd)]
    del full
    split = shard_sizes(gs[dd], n)
    outs = [torch.empty(1, 65536, split[k], 128, dtype=torch.bfloat16, device="cuda:0") for k in range(n)]
    in_shape = list(shards[0].shape)

    def body(comm, r, s):
        comm.all_to_all(r, shards[r].data_ptr(), outs[r].data_ptr(), in_shape, sd, dd, src_lens, 2, s.cuda_stream)

    _same_device(n, body)
    host = [raw_from_torch(t) for t in shards]
    want = R.all_to_all(host, sd, dd)
    for k in range(n):
        assert np.array_equal(np_raw(outs[k]).reshape(want[k].shape), want[k]), k
    if Reference.available():
        ref_outs, _ = Reference().all_to_all(host, 1, sd, dd)
        for k in range(n):
            assert np.array_equal(np_raw(outs[k]).reshape(want[k].shape), ref_outs[k]), k
