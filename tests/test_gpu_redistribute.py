"""GPU: the reference-facing host layer -- ThreadGroup (the reference's communicator API) and
DTensor.redistribute -- on the B200 collectives, on the cases of the reference's own tests:

* dtorch/tests/test_nccl.cc:27-45: one thread per rank, ThreadGroup.AllReduce of ones == group size.
* python/dtorch/test/test_distributed_tensor.py:146-393: 1-D mesh [0, 1] with even (4, 8) and uneven (5, 9)
  shapes (P->R, P->S0, S0->R, S1->R, S1->S0, S0->S1, R->S1), 2-D mesh (4, 2), 3-D mesh (2, 2, 2).

Each runs in the reference's two modes: same-device emulation (DTORCH_DTENSOR_IN_SAME_DEVICE=1: every rank
on cuda:0, one kernel per collective) and peer mode (rank r on cuda:r) when enough GPUs are present. Results
are compared with the whole tensor (as the reference does, allclose rtol 1e-5 / atol 1e-8 -- here
bit-exact, since moves are copies and the fp32 sums fold in the reference's order), and sums with the
oracle fold.
"""

import math
import os
import threading

import numpy as np
import pytest
import torch

import dtorch_b200 as dtb
from oracle.oracle import Restatement

pytestmark = pytest.mark.gpu
R = Restatement()


def ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture(params=["same", "peer"])
def mode(request):
    if ngpu() < 1:
        pytest.skip("no CUDA device")
    old = os.environ.get("DTORCH_DTENSOR_IN_SAME_DEVICE")
    if request.param == "same":
        os.environ["DTORCH_DTENSOR_IN_SAME_DEVICE"] = "1"
    else:
        os.environ.pop("DTORCH_DTENSOR_IN_SAME_DEVICE", None)
    os.environ.setdefault("DTORCH_COMM_TIMEOUT_SECOND", "30")
    dtb.clear()
    yield request.param
    dtb.clear()
    if old is None:
        os.environ.pop("DTORCH_DTENSOR_IN_SAME_DEVICE", None)
    else:
        os.environ["DTORCH_DTENSOR_IN_SAME_DEVICE"] = old


def need(mode, n):
    if mode == "peer" and ngpu() < n:
        pytest.skip(f"peer mode on {n} devices needs {n} GPUs")


def test_thread_group_all_reduce_of_ones(mode):
    n = 2 if mode == "same" or ngpu() < 8 else 8
    need(mode, n)
    ids = list(range(n))
    results = [None] * n
    errors = []

    def rank_fn(r):
        try:
            dev = dtb.cuda_device_of(r)
            with torch.cuda.device(dev):
                tg = dtb.dtensor._host.get_thread_group(ids, r)
                assert tg.get_rank() == r and tg.get_world_size() == n and tg.get_global_device_id() == r
                x = torch.ones(1000, 1000, device=f"cuda:{dev}")
                tg.barrier()
                y = tg.all_reduce(x)
                tg.barrier()
                torch.cuda.current_stream(dev).synchronize()
                results[r] = y
        except BaseException as e:  # noqa: BLE001
            errors.append(e)

    th = [threading.Thread(target=rank_fn, args=(r,)) for r in range(n)]
    for t in th:
        t.start()
    for t in th:
        t.join(60)
    assert not errors, errors
    for y in results:
        assert torch.equal(y.cpu(), torch.full((1000, 1000), float(n)))


def check_redistribute(mesh, full, src, dst, expected=None):
    x = dtb.DTensor.from_torch(full, mesh, src)
    y = x.redistribute(device_mesh=mesh, placements=dst)
    torch.cuda.synchronize()
    got = y.to_torch()
    want = full if expected is None else expected
    assert got.shape == want.shape
    assert torch.equal(got, want), f"{src} -> {dst}"
    return y


@pytest.mark.parametrize("shape", [(4, 8), (5, 9)])
def test_redistribute_1d_like_reference(mode, shape):
    need(mode, 2)
    g = torch.Generator().manual_seed(0)
    full = torch.rand(*shape, generator=g)
    mesh = dtb.DeviceMesh("cuda", [0, 1])
    S, Rp, P = dtb.Shard, dtb.Replicate, dtb.Partial
    # Partial built as the reference builds it: the tensor on rank 0, zeros elsewhere
    check_redistribute(mesh, full, [P()], [Rp()])
    if shape[0] % 2 == 0:
        y = check_redistribute(mesh, full, [P()], [S(0)])
        assert y.local(0).shape == (shape[0] // 2, shape[1])
    check_redistribute(mesh, full, [S(0)], [Rp()])
    check_redistribute(mesh, full, [S(-1)], [Rp()])
    check_redistribute(mesh, full, [S(-1)], [S(0)])
    check_redistribute(mesh, full, [S(0)], [S(1)])
    check_redistribute(mesh, full, [Rp()], [S(1)])
    # local shapes follow the shard rule
    y = dtb.DTensor.from_torch(full, mesh, [S(1)])
    assert y.local(0).shape[1] == (shape[1] + 1) // 2 and y.local(1).shape[1] == shape[1] // 2


def test_redistribute_partial_sum_matches_oracle(mode):
    need(mode, 4)
    n = 4
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(1)
    parts = [torch.randn(64, 33, generator=g) for _ in range(n)]
    locals_ = {r: parts[r].to(f"cuda:{dtb.cuda_device_of(r)}") for r in range(n)}
    x = dtb.DTensor(locals_, mesh, [dtb.Partial()], (64, 33))
    want = R.fold_sum([p.numpy() for p in parts], 0, storage_round=True)
    y = x.redistribute(placements=[dtb.Replicate()])
    torch.cuda.synchronize()
    for r in range(n):
        assert np.array_equal(y.local(r).cpu().numpy(), want)
    z = x.redistribute(placements=[dtb.Shard(0)])
    torch.cuda.synchronize()
    assert np.array_equal(z.to_torch().numpy(), want)


def test_redistribute_2d_like_reference(mode):
    need(mode, 8)
    mesh = dtb.init_device_mesh("cuda", (4, 2))
    g = torch.Generator().manual_seed(2)
    full = torch.rand(4, 16, generator=g)
    S, Rp = dtb.Shard, dtb.Replicate
    check_redistribute(mesh, full, [S(0), S(1)], [Rp(), S(1)])
    check_redistribute(mesh, full, [S(0), S(1)], [S(0), Rp()])
    check_redistribute(mesh, full, [Rp(), Rp()], [S(1), Rp()])
    check_redistribute(mesh, full, [Rp(), Rp()], [S(1), S(1)])
    check_redistribute(mesh, full, [S(0), S(1)], [Rp(), Rp()])


def test_redistribute_3d_like_reference(mode):
    need(mode, 8)
    mesh = dtb.init_device_mesh("cuda", (2, 2, 2))
    g = torch.Generator().manual_seed(3)
    full = torch.rand(2, 16, 128, 128, generator=g)
    S, Rp = dtb.Shard, dtb.Replicate
    check_redistribute(mesh, full, [S(0), S(2), S(2)], [Rp(), Rp(), Rp()])
    check_redistribute(mesh, full, [Rp(), Rp(), Rp()], [S(0), S(2), S(2)])


@pytest.mark.parametrize("n", [2, 4, 8])
def test_ulysses_swap_and_back(mode, n):
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(n)
    full = torch.randn(1, 96, 12, 16, generator=g).to(torch.bfloat16)  # (B, S, H, D); uneven heads at n=8
    x = dtb.DTensor.from_torch(full, mesh, [dtb.Shard(1)])
    y = x.redistribute(placements=[dtb.Shard(2)])  # sequence-sharded -> head-sharded
    z = y.redistribute(placements=[dtb.Shard(1)])  # and back
    torch.cuda.synchronize()
    assert torch.equal(y.to_torch(), full)
    assert torch.equal(z.to_torch(), full)
    for r in range(n):
        assert torch.equal(z.local(r).cpu(), x.local(r).cpu())


@pytest.mark.parametrize("n", [2, 4])
def test_fused_qkv_all_to_all_matches_separate(mode, n):
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(10 + n)
    fulls = [torch.randn(2, 8, 40, 16, generator=g).to(torch.bfloat16) for _ in range(3)]  # (N, H, L, E)
    xs = [dtb.DTensor.from_torch(f, mesh, [dtb.Shard(2)]) for f in fulls]
    fused = dtb.redistribute_many(xs, [dtb.Shard(1)])
    torch.cuda.synchronize()
    for x, y, f in zip(xs, fused, fulls):
        sep = x.redistribute(placements=[dtb.Shard(1)])
        torch.cuda.synchronize()
        for r in range(n):
            assert torch.equal(y.local(r).cpu(), sep.local(r).cpu())
        assert torch.equal(y.to_torch(), f)


@pytest.mark.parametrize("is_causal", [False, True])
def test_ulysses_attention_matches_torch(mode, is_causal):
    n = 4
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,), mesh_dim_names=["cp"])
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 8, 64, 32, generator=g) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda(), is_causal=is_causal).cpu()
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, is_causal=is_causal, ulysses_cp_dim="cp")
    torch.cuda.synchronize()
    assert out.placements == [dtb.Shard(2)]
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


def test_ring_attention_matches_torch(mode):
    n = 2
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(1, 4, 48, 16, generator=g) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, ring_cp_dim=0)
    torch.cuda.synchronize()
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("shape,placements,dims", [
    ((8, 6), ["S0"], [0]),
    ((9, 7, 4), ["S1"], [1, 2]),
    ((6, 10), ["S1"], [0]),          # reduce a dim that is not sharded: no communication
    ((4, 12, 5), ["S2"], [0, 2]),
])
def test_reduce_over_sharded_dims(mode, shape, placements, dims):
    need(mode, 2)
    mesh = dtb.DeviceMesh("cuda", [0, 1])
    g = torch.Generator().manual_seed(5)
    full = torch.randn(*shape, generator=g)
    x = dtb.DTensor.from_torch(full, mesh, [dtb.Placement(p) for p in placements])
    for kind in ("sum", "mean"):
        for keepdim in (False, True):
            y = dtb.reduce(x, dims, kind=kind, keepdim=keepdim)
            torch.cuda.synchronize()
            want = full.sum(dim=dims, keepdim=keepdim) if kind == "sum" else full.mean(dim=dims, keepdim=keepdim)
            assert tuple(y.shape) == tuple(want.shape)
            assert torch.allclose(y.to_torch(), want, rtol=1e-5, atol=1e-5), (kind, keepdim)


@pytest.mark.parametrize("n,length,sub", [(2, 6, 2), (2, 9, 4), (4, 16, 7), (4, 19, 5)])
def test_sub_split_shard_round_trip(mode, n, length, sub):
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(length + sub)
    full = torch.randn(3, length, 5, generator=g)
    ss = dtb.Shard(1, sub)
    x = dtb.DTensor.from_torch(full, mesh, [ss])
    assert torch.equal(x.to_torch(), full)
    r = x.redistribute(placements=[dtb.Replicate()])  # all-gather into pieces + sub-split reassembly
    torch.cuda.synchronize()
    for gid in range(n):
        assert torch.equal(r.local(gid).cpu(), full)
    back = r.redistribute(placements=[ss])  # local sub-split slicing
    torch.cuda.synchronize()
    for gid in range(n):
        assert torch.equal(back.local(gid).cpu(), x.local(gid).cpu())


def test_redistribute_to_another_mesh(mode):
    # pipeline-stage handoff: mesh [0, 1] -> mesh [2, 3] (peer mode needs 4 GPUs), optionally changing placements
    need(mode, 4)
    a = dtb.DeviceMesh("cuda", [0, 1])
    b = dtb.DeviceMesh("cuda", [2, 3])
    g = torch.Generator().manual_seed(8)
    full = torch.randn(6, 10, generator=g)
    x = dtb.DTensor.from_torch(full, a, [dtb.Shard(0)])
    y = x.redistribute(device_mesh=b)
    z = x.redistribute(device_mesh=b, placements=[dtb.Shard(1)])
    torch.cuda.synchronize()
    assert y.device_mesh == b and y.placements == [dtb.Shard(0)]
    assert torch.equal(y.to_torch(), full) and torch.equal(z.to_torch(), full)
    assert z.placements == [dtb.Shard(1)]
    for dst in (2, 3):
        assert y.local(dst).device.index == dtb.cuda_device_of(dst)


def test_ring_attention_causal_as_reference(mode):
    # the reference runs torch's attention per device on its query chunk against the gathered K/V with
    # is_causal=True (SdpaOp::Compute): the result is that, chunk by chunk
    n = 2
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(6)
    q, k, v = (torch.randn(1, 4, 48, 16, generator=g) for _ in range(3))
    chunks = torch.split(q, dtb.dtensor._host.shard_sizes(48, n), 2)
    want = torch.cat([torch.nn.functional.scaled_dot_product_attention(c.cuda(), k.cuda(), v.cuda(),
                                                                       is_causal=True).cpu() for c in chunks], 2)
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, is_causal=True, ring_cp_dim=0)
    torch.cuda.synchronize()
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("cp", ["ring", "ulysses"])
def test_attention_on_sub_split_sequence(mode, cp):
    # non-causal: sub-split sequence shards are viewed as Shard(2) for the call and the output viewed back
    n = 2
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,), mesh_dim_names=["cp"])
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 4, 40, 16, generator=g) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    ss = dtb.Shard(2, 13)
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [ss]) for t in (q, k, v))
    kw = {"ring_cp_dim": "cp"} if cp == "ring" else {"ulysses_cp_dim": "cp"}
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, **kw)
    torch.cuda.synchronize()
    assert out.placements == [ss]
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("n,S", [(2, 45), (4, 64)])
def test_ring_attention_overlapped_matches_torch(mode, n, S):
    # own-chunk attention during the K/V all-gather, other chunks after, merged by log-sum-exp
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,), mesh_dim_names=["ring"])
    g = torch.Generator().manual_seed(S)
    q, k, v = (torch.randn(2, 4, S, 16, generator=g) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, ring_cp_dim="ring", ring_overlap=True)
    torch.cuda.synchronize()
    assert out.placements == [dtb.Shard(2)]
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


def test_ring_attention_overlapped_bf16(mode):
    n = 2
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,))
    g = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn(1, 8, 96, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.float().cuda(), k.float().cuda(), v.float().cuda()).cpu()
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, ring_cp_dim=0, ring_overlap=True)
    torch.cuda.synchronize()
    got = out.to_torch().float()
    assert got.dtype == torch.float32 and out.dtype == torch.bfloat16
    assert torch.allclose(got, want, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("overlap", [False, True])
def test_ulysses_and_ring_attention_on_2d_mesh(mode, overlap):
    need(mode, 4)
    mesh = dtb.init_device_mesh("cuda", (2, 2), mesh_dim_names=["u", "r"])
    g = torch.Generator().manual_seed(14)
    q, k, v = (torch.randn(1, 4, 48, 16, generator=g) for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    pl = [dtb.Shard(2), dtb.Shard(2)]
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, pl) for t in (q, k, v))
    out = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, ulysses_cp_dim="u", ring_cp_dim="r",
                                                   ring_overlap=overlap)
    torch.cuda.synchronize()
    assert out.placements == pl
    assert torch.allclose(out.to_torch(), want, rtol=1e-4, atol=1e-5)


def test_redistribute_by_dict(mode):
    # python/dtorch/tensor.py:317-351: placements by mesh dim name, the rest kept; a shard of a size-1 dim becomes
    # Replicate
    need(mode, 4)
    mesh = dtb.init_device_mesh("cuda", (2, 2), mesh_dim_names=["dp", "tp"])
    g = torch.Generator().manual_seed(15)
    full = torch.randn(1, 12, 10, generator=g)
    x = dtb.DTensor.from_torch(full, mesh, [dtb.Shard(1), dtb.Shard(2)])
    y = x.redistribute_by_dict(placements_dict={"tp": dtb.Replicate()}, default_placement_mode="keep")
    z = x.redistribute_by_dict(placements_dict={"dp": dtb.Shard(0), "tp": dtb.Shard(2)})
    torch.cuda.synchronize()
    assert y.placements == [dtb.Shard(1), dtb.Replicate()]
    assert z.placements == [dtb.Replicate(), dtb.Shard(2)]  # Shard(0) of a size-1 dim -> Replicate
    assert torch.equal(y.to_torch(), full) and torch.equal(z.to_torch(), full)


@pytest.mark.parametrize("mesh_shape", [(2, 2, 2), (2, 1, 2)])
def test_redistribute_by_dim_name_like_reference(mode, mesh_shape):
    # python/dtorch/test/test_distributed_tensor.py:408-439
    need(mode, math.prod(mesh_shape))
    mesh = dtb.init_device_mesh("cuda", mesh_shape, mesh_dim_names=["dp", "cp", "tp"])
    g = torch.Generator().manual_seed(16)
    full = torch.rand(2, 4, 8, generator=g)
    x = dtb.DTensor.from_torch(full, mesh, [dtb.Replicate()] * 3)
    y = x.redistribute_by_dict(placements_dict={"dp": dtb.Shard(0), "cp": dtb.Shard(1), "tp": dtb.Shard(1)})
    torch.cuda.synchronize()
    assert torch.equal(y.to_torch(), full)
    cp = dtb.Shard(1) if mesh_shape[1] > 1 else dtb.Replicate()
    assert y.placements == [dtb.Shard(0), cp, dtb.Shard(1)]


def test_mesh_move_between_two_gpus_by_peer_copy_kernel(mode):
    # mesh [0, 1] -> mesh [1, 0]: every local crosses to the other GPU (same-device mode: stays on cuda:0)
    need(mode, 2)
    from dtorch_b200 import capi

    a = dtb.DeviceMesh("cuda", [0, 1])
    b = dtb.DeviceMesh("cuda", [1, 0])
    g = torch.Generator().manual_seed(21)
    full = torch.randn(9, 1000 + 3, generator=g).to(torch.bfloat16)  # odd rows: 4-byte-aligned runs
    x = dtb.DTensor.from_torch(full, a, [dtb.Shard(0)])
    n0 = capi.launch_count()
    y = x.redistribute(device_mesh=b)
    for d in range(min(2, ngpu())):
        torch.cuda.synchronize(d)
    if mode == "peer":
        assert capi.launch_count() - n0 == 2, "one peer-copy kernel per local"
    assert torch.equal(y.to_torch(), full)
    assert torch.equal(y.local(1).cpu(), x.local(0).cpu()) and torch.equal(y.local(0).cpu(), x.local(1).cpu())
    # a whole DTensor gathered onto one GPU
    tgt = 1 if mode == "peer" else 0
    on_gpu = x.to_torch(device=f"cuda:{tgt}")
    assert on_gpu.device.index == tgt
    assert torch.equal(on_gpu.cpu(), full)


@pytest.mark.parametrize("nbytes,src_off,dst_off", [(1, 0, 0), (4097, 3, 5), ((64 << 20) + 16, 0, 0), (1000003, 16, 48)])
def test_peer_copy_c_abi(nbytes, src_off, dst_off):
    if ngpu() < 2:
        pytest.skip("needs 2 GPUs")
    from dtorch_b200 import capi

    src = torch.randint(0, 255, (nbytes + src_off,), dtype=torch.uint8, device="cuda:0")
    dst = torch.zeros(nbytes + dst_off + 7, dtype=torch.uint8, device="cuda:1")
    s = torch.cuda.current_stream(0)
    s.wait_stream(torch.cuda.current_stream(1))
    capi.peer_copy(dst.data_ptr() + dst_off, 1, src.data_ptr() + src_off, 0, nbytes, s.cuda_stream)
    s.synchronize()
    got = dst.cpu()
    assert torch.equal(got[dst_off:dst_off + nbytes], src.cpu()[src_off:])
    assert int(got[:dst_off].sum()) == 0 and int(got[dst_off + nbytes:].sum()) == 0


@pytest.mark.parametrize("groups", [2, 4])
@pytest.mark.parametrize("is_causal", [False, True])
def test_ulysses_overlapped_equals_plain(mode, groups, is_causal):
    n = 2
    need(mode, n)
    mesh = dtb.init_device_mesh("cuda", (n,), mesh_dim_names=["cp"])
    g = torch.Generator().manual_seed(31)
    q, k, v = (torch.randn(1, 16, 96, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    dq, dk, dv = (dtb.DTensor.from_torch(t, mesh, [dtb.Shard(2)]) for t in (q, k, v))
    plain = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, is_causal=is_causal, ulysses_cp_dim="cp")
    piped = dtb.scaled_dot_product_attention_with_cp(dq, dk, dv, is_causal=is_causal, ulysses_cp_dim="cp",
                                                     ulysses_overlap_groups=groups)
    for d in range(min(n, ngpu())):
        torch.cuda.synchronize(d)
    assert piped.placements == plain.placements
    for gid in mesh.ids:
        assert torch.equal(piped.local(gid).cpu(), plain.local(gid).cpu()), gid
