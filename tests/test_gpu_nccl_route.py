"""GPU: the all-reduce routed to NCCL where NCCL measured faster than the rank-order kernels.

DTorch's own GPU backend is NCCL (ThreadGroup's constructor picks it for distinct devices,
dtorch/core/communication/thread_group/thread_group.cc:75-88); here NCCL is one algorithm of dt_all_reduce, used
for ordinary buffers at 8 ranks from 256 MiB (or forced with DT_ALGO_NCCL), on a clique of NCCL communicators
the library makes over the communicator's devices. Checked here:

* forced: every rank holds the same result, within the reductions' tolerance of the rank-order fold (NCCL sums
  in its own order), and none of this library's kernels runs;
* the default choice: from 256 MiB at 8 ranks the call goes to NCCL; just below, with DT_RANK_ORDER, or with
  DTORCH_B200_NCCL=0 the rank-order two-shot kernel runs; integer-valued fp32 partials make every summation
  order exact, so all of them are compared bit for bit;
* the forms that are rejected before any work: same-device mode, DT_ACCUM_STORAGE, combined algorithm bits.
"""

import threading

import numpy as np
import pytest
import torch

from dtorch_b200 import capi
from oracle.oracle import Restatement
from tests.gpu_util import np_raw, run_ranks
from tests.helpers import DT_CODE, abs_sum_f64, assert_close_sum, raw_from_torch

pytestmark = pytest.mark.gpu
R = Restatement()


def ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture(autouse=True)
def _need_gpu():
    if ngpu() < 1:
        pytest.skip("no CUDA device")


def _counted_all_reduce(comm, n, xs, ys, count, code, flags):
    """Every rank thread calls dt_all_reduce once; returns how many of this library's kernels the call launched
    (counted between barriers, with every rank's stream idle on both sides)."""
    bar = threading.Barrier(n)
    counts = {}

    def fn(r):
        with torch.cuda.device(r):
            st = torch.cuda.current_stream(r)
            st.synchronize()
            bar.wait(timeout=120)
            if r == 0:
                counts["a"] = capi.launch_count()
            bar.wait(timeout=120)
            comm.all_reduce(r, xs[r].data_ptr(), ys[r].data_ptr(), count, code, flags, st.cuda_stream)
            st.synchronize()
            bar.wait(timeout=120)
            if r == 0:
                counts["b"] = capi.launch_count()

    run_ranks(n, fn)
    return counts["b"] - counts["a"]


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
def test_forced_nccl_all_reduce(dt):
    n = min(ngpu(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    td = torch.float32 if dt == "float32" else torch.bfloat16
    count = (1 << 20) + 5
    comm = capi.Comm(list(range(n)))
    try:
        g = torch.Generator().manual_seed(77)
        host = [torch.randn(count, generator=g).to(td) for _ in range(n)]
        xs = [h.to(f"cuda:{r}") for r, h in enumerate(host)]
        ys = [torch.empty_like(x) for x in xs]
        for _ in range(2):  # the first call makes the clique, the second reuses it
            launched = _counted_all_reduce(comm, n, xs, ys, count, DT_CODE[dt], capi.DT_ALGO_NCCL)
            assert launched == 0, "NCCL ran the reduction, not this library's kernels"
        got = [np_raw(y) for y in ys]
        raw = [raw_from_torch(h) for h in host]
        want = R.fold_sum(raw, DT_CODE[dt], storage_round=False)
        for r in range(n):
            assert np.array_equal(got[r], got[0]), "every rank holds the same sum"
        assert_close_sum(got[0], want, dt, abs_sum_f64(raw, dt))
        # the same communicator still runs the rank-order kernels afterwards
        launched = _counted_all_reduce(comm, n, xs, ys, count, DT_CODE[dt], capi.DT_ALGO_TWOSHOT)
        assert launched == n
        for r in range(n):
            assert np.array_equal(np_raw(ys[r]), want), r
    finally:
        comm.destroy()


def test_default_choice_routes_to_nccl_at_8_ranks_from_256_MiB(monkeypatch):
    if ngpu() < 8:
        pytest.skip("the NCCL route is taken at 8 ranks")
    n = 8
    count = (256 << 20) // 4  # fp32: exactly the switch-over size
    xs, ys = [], []
    for r in range(n):
        g = torch.Generator(device=f"cuda:{r}").manual_seed(r)
        xs.append(torch.randint(-64, 65, (count,), generator=g, device=f"cuda:{r}").to(torch.float32))
        ys.append(torch.empty_like(xs[r]))
    want = xs[0].clone()
    for r in range(1, n):
        want += xs[r].to("cuda:0")  # integers: exact in every order

    def check(prefix):
        for r in range(n):
            assert torch.equal(ys[r][:prefix].to("cuda:0"), want[:prefix]), r

    comm = capi.Comm(list(range(n)))
    try:
        assert _counted_all_reduce(comm, n, xs, ys, count, capi.DT_FLOAT32, 0) == 0  # NCCL
        check(count)
        assert _counted_all_reduce(comm, n, xs, ys, count - 4, capi.DT_FLOAT32, 0) == n  # 16 bytes short
        check(count - 4)
        assert _counted_all_reduce(comm, n, xs, ys, count, capi.DT_FLOAT32, capi.DT_RANK_ORDER) == n
        check(count)
    finally:
        comm.destroy()
    monkeypatch.setenv("DTORCH_B200_NCCL", "0")
    comm = capi.Comm(list(range(n)))
    try:
        assert _counted_all_reduce(comm, n, xs, ys, count, capi.DT_FLOAT32, 0) == n
        check(count)
    finally:
        comm.destroy()


def test_nccl_forms_rejected_before_any_work():
    comm = capi.Comm([0, 0])  # same-device mode: rejected before the ranks' rendezvous
    try:
        x = torch.zeros(16, device="cuda:0")
        cases = [(capi.DT_ALGO_NCCL, capi.DT_ERR_UNSUPPORTED),
                 (capi.DT_ALGO_NCCL | capi.DT_ACCUM_STORAGE, capi.DT_ERR_UNSUPPORTED),
                 (capi.DT_ALGO_NCCL | capi.DT_RANK_ORDER, capi.DT_ERR_UNSUPPORTED),
                 (capi.DT_ALGO_NCCL | capi.DT_ALGO_TWOSHOT, capi.DT_ERR_INVALID)]
        for flags, status in cases:
            with pytest.raises(capi.DtError) as e:
                comm.all_reduce(0, x.data_ptr(), x.data_ptr(), 16, capi.DT_FLOAT32, flags)
            assert e.value.status == status, flags
    finally:
        comm.destroy()
