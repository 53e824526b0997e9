"""GPU test of dt_local_all_reduce_host_noalloc, the host-partials all-reduce for callers that cannot allocate
device memory (a caller holding host tensors only, or one whose GPU memory another allocator owns): it stages
through the library's fixed device scratch instead of buffers the caller passes in.

Its results must equal those of dt_local_all_reduce_host, the entry point with caller-provided staging, on the
same partials -- bit for bit, the tolerance the reduction tests use against the fp32-accumulate fold -- on two
calls in a row, the second of which reuses the scratch the first one left behind. The file is named so pytest
collects it last; it also passes on its own in a fresh process.
"""

import numpy as np
import pytest
import torch

from dtorch_b200 import capi
from oracle.oracle import Restatement
from tests.helpers import DT_CODE, raw_from_torch

pytestmark = pytest.mark.gpu
R = Restatement()
TD = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _with_staging(host, count, code, flags, stream):
    """The same all-reduce through dt_local_all_reduce_host, with staging buffers allocated here."""
    td = host[0].dtype
    dev = [torch.empty(count, dtype=td, device="cuda:0") for _ in host]
    dout = torch.empty(count, dtype=td, device="cuda:0")
    hout = torch.empty(count, dtype=td).pin_memory()
    capi.local_all_reduce_host([h.data_ptr() for h in host], [d.data_ptr() for d in dev], dout.data_ptr(),
                               hout.data_ptr(), count, code, flags, 0, stream.cuda_stream)
    stream.synchronize()
    return raw_from_torch(hout)


@pytest.mark.parametrize("dt,n,count,flags", [
    ("bfloat16", 8, 1_000_003, 0),
    ("float32", 4, 300_001, 0),
    ("float16", 3, 77_777, capi.DT_ACCUM_STORAGE),
])
def test_noalloc_matches_staged_entry_point_twice(dt, n, count, flags):
    torch.cuda.set_device(0)
    code, td = DT_CODE[dt], TD[dt]
    stream = torch.cuda.Stream(device=0)
    g = torch.Generator().manual_seed(1234 + n)
    for call in range(2):  # the second call finds the first call's contents in the scratch
        host = [torch.randn(count, generator=g).to(td).pin_memory() for _ in range(n)]
        hout = torch.full((count,), float("nan"), dtype=td).pin_memory()
        before = capi.launch_count()
        capi.local_all_reduce_host_noalloc([h.data_ptr() for h in host], hout.data_ptr(), count, code, flags,
                                           stream.cuda_stream)
        stream.synchronize()
        assert capi.launch_count() - before == 1, "one reduction kernel per call"
        got = raw_from_torch(hout)
        want = _with_staging(host, count, code, flags, stream)
        assert np.array_equal(got, want), f"call {call}: differs from dt_local_all_reduce_host"
        assert np.array_equal(got, R.fold_sum([raw_from_torch(h) for h in host], code, flags == capi.DT_ACCUM_STORAGE))


def test_noalloc_rejects_more_than_the_scratch_holds():
    torch.cuda.set_device(0)
    n, es = 8, 2
    slot_limit = capi.NOALLOC_SCRATCH_BYTES // (n + 1) // 256 * 256
    ok_count = slot_limit // es
    too_big = ok_count + 256
    host = [torch.zeros(too_big, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    hout = torch.empty(too_big, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(capi.DtError) as e:
        capi.local_all_reduce_host_noalloc([h.data_ptr() for h in host], hout.data_ptr(), too_big, capi.DT_BFLOAT16)
    assert e.value.status == capi.DT_ERR_INVALID
    assert "static scratch holds" in str(e.value)
    # the largest size that fits still runs
    stream = torch.cuda.Stream(device=0)
    for h in host:
        h[:ok_count].fill_(1.0)
    capi.local_all_reduce_host_noalloc([h.data_ptr() for h in host], hout.data_ptr(), ok_count, capi.DT_BFLOAT16, 0,
                                       stream.cuda_stream)
    stream.synchronize()
    assert torch.equal(hout[:ok_count], torch.full((ok_count,), float(n), dtype=torch.bfloat16))
