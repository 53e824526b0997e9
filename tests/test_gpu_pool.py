"""GPU: the symmetric pool behind DTensor locals and ThreadGroup outputs (peer mode, one process, >= 2 GPUs).

With a pool, from_torch places every device's local at the same offset of the group's peer-mapped memory and
every collective allocates its outputs there too, so the collectives resolve peers without the per-call
pointer exchange; on NVLink-multicast GPUs the pool is the NVLS buffer and all-reduces of 8 MiB and more at
>= 6 ranks reduce in the switch. Results are checked against the oracle as everywhere else (bit-exact for
moves and rank-order folds; NVLS within the reductions' tolerance).
"""

import os

import numpy as np
import pytest
import torch

import dtorch_b200 as dtb
from oracle.oracle import Restatement
from tests.helpers import abs_sum_f64, assert_close_sum, raw_from_torch

pytestmark = pytest.mark.gpu
R = Restatement()


def ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture
def pool():
    if ngpu() < 2:
        pytest.skip("the symmetric pool serves peer groups: needs >= 2 GPUs")
    old = os.environ.pop("DTORCH_DTENSOR_IN_SAME_DEVICE", None)
    os.environ.setdefault("DTORCH_COMM_TIMEOUT_SECOND", "30")
    dtb.clear()
    dtb.set_pool_bytes(256 << 20)
    yield
    dtb.clear()
    dtb.set_pool_bytes(0)
    if old is not None:
        os.environ["DTORCH_DTENSOR_IN_SAME_DEVICE"] = old


def _in_pool(mesh, t, gid):
    return dtb.dtensor._host.in_pool(mesh.ids, gid, t)


@pytest.mark.parametrize("n", [2, 4, 8])
def test_pool_collectives_stay_in_pool_and_match_oracle(pool, n):
    if ngpu() < n:
        pytest.skip(f"needs {n} GPUs")
    mesh = dtb.DeviceMesh("cuda", list(range(n)))
    g = torch.Generator().manual_seed(n)
    full = torch.randn(64 * n + 3, 96, generator=g)
    # S0 -> R (uneven shards), R -> S1, S1 -> S0, P -> R, P -> S0: every local and output in the pool
    x = dtb.DTensor.from_torch(full, mesh, [dtb.Shard(0)])
    assert all(_in_pool(mesh, x.local(i), i) for i in mesh.ids)
    y = x.redistribute(placements=[dtb.Replicate()])
    assert all(_in_pool(mesh, y.local(i), i) for i in mesh.ids)
    torch.cuda.synchronize()
    assert torch.equal(y.to_torch(), full)
    z = y.redistribute(placements=[dtb.Shard(1)]).redistribute(placements=[dtb.Shard(0)])
    torch.cuda.synchronize()
    assert torch.equal(z.to_torch(), full)
    parts = [torch.randn(256, 1024, generator=g) for _ in range(n)]
    p = dtb.DTensor.empty({i: (256, 1024) for i in mesh.ids}, torch.float32, mesh, [dtb.Partial()], (256, 1024))
    for i in mesh.ids:
        p.local(i).copy_(parts[i])
    torch.cuda.synchronize()
    want = R.fold_sum([t.numpy().reshape(-1) for t in parts], 0, storage_round=False)
    r = p.redistribute(placements=[dtb.Replicate()])
    s = p.redistribute(placements=[dtb.Shard(0)])
    torch.cuda.synchronize()
    for i in mesh.ids:
        assert _in_pool(mesh, r.local(i), i) and _in_pool(mesh, s.local(i), i)
        assert np.array_equal(r.local(i).cpu().numpy().reshape(-1), want)
    assert np.array_equal(s.to_torch().numpy().reshape(-1), want)


def test_pool_nvls_all_reduce_within_tolerance(pool):
    n = min(ngpu(), 8)
    if n < 6:
        pytest.skip("the NVLS all-reduce is chosen at >= 6 ranks")
    mesh = dtb.DeviceMesh("cuda", list(range(n)))
    info = dtb.dtensor._host.pool_info(mesh.ids, 0)
    if not info["nvls"]:
        pytest.skip("no NVLink multicast on these GPUs")
    shape = (2048, 8192)  # 32 MiB of bf16 per rank: above the NVLS threshold
    p = dtb.DTensor.empty({i: shape for i in mesh.ids}, torch.bfloat16, mesh, [dtb.Partial()], shape)
    host = []
    for i in mesh.ids:
        t = torch.randn(shape, generator=torch.Generator().manual_seed(i)).to(torch.bfloat16)
        host.append(raw_from_torch(t))
        p.local(i).copy_(t)
    torch.cuda.synchronize()
    r = p.redistribute(placements=[dtb.Replicate()])
    torch.cuda.synchronize()
    want = R.fold_sum(host, 1, storage_round=False)
    scale = abs_sum_f64(host, "bfloat16")
    first = raw_from_torch(r.local(0))
    for i in mesh.ids:
        got = raw_from_torch(r.local(i))
        assert np.array_equal(got, first), "every rank holds the same NVLS result"
        assert_close_sum(got, want, "bfloat16", scale)


def test_pool_reuse_and_exhaustion(pool):
    n = 2
    mesh = dtb.DeviceMesh("cuda", list(range(n)))
    info = dtb.dtensor._host.pool_info(mesh.ids, 0)
    assert info["bytes"] >= 256 << 20
    g = torch.Generator().manual_seed(3)
    # many rounds of alloc / free: blocks come back once the GPU is done with them
    for k in range(20):
        full = torch.randn(4096, 1024, generator=g)  # 16 MiB per replica
        x = dtb.DTensor.from_torch(full, mesh, [dtb.Shard(0)])
        y = x.redistribute(placements=[dtb.Replicate()])
        torch.cuda.synchronize()
        assert torch.equal(y.to_torch(), full), k
        del x, y
    torch.cuda.synchronize()
    # a request larger than the pool falls back to ordinary allocations on every rank, still correct
    big = torch.randn(16384, 8192, generator=g)  # 512 MiB replicated
    x = dtb.DTensor.from_torch(big, mesh, [dtb.Shard(0)])
    y = x.redistribute(placements=[dtb.Replicate()])
    torch.cuda.synchronize()
    assert not _in_pool(mesh, y.local(0), 0)
    assert torch.equal(y.to_torch(), big)
    del x, y
    torch.cuda.synchronize()
    import gc

    gc.collect()
    torch.cuda.synchronize()
    dtb.dtensor._host.pool_info(mesh.ids, 0)  # reclaims finished blocks
