"""CPU: the placement algebra of the host layer (dtorch_b200/csrc/host/placement.cpp) against the reference's
rules, on cases worked out from dtorch/api/cpp/distributed_spec.cc and thread_group_manager.cc."""

import pytest

h = pytest.importorskip("dtorch_b200._host")


def test_shard_sizes():
    assert h.shard_sizes(9, 2) == [5, 4]
    assert h.shard_sizes(17, 8) == [3, 2, 2, 2, 2, 2, 2, 2]
    assert h.shard_sizes(65536, 8) == [8192] * 8


def test_convert_order_shard_to_replicate_last_back_to_front():
    # distributed_spec.cc:327-343: changed dims in order, then S->R dims reversed
    assert h.get_convert_order(["S0", "S1", "P"], ["R", "R", "R"]) == [2, 1, 0]
    assert h.get_convert_order(["S0", "R"], ["R", "S1"]) == [1, 0]
    assert h.get_convert_order(["S0", "S2", "S2"], ["R", "R", "R"]) == [2, 1, 0]
    assert h.get_convert_order(["R", "R"], ["S1", "S1"]) == [0, 1]
    assert h.get_convert_order(["R"], ["R"]) == []
    assert h.get_diff_dims(["S0", "S1"], ["R", "S1"]) == [0]


def test_normalize():
    assert h.normalize(["S-1"], [2], [0, 1], 2) == ["S1"]
    assert h.normalize(["S0", "S1", "P"], [2, 1, 4], list(range(8)), 3) == ["S0", "R", "P"]


def test_group_device_ids():
    ids = list(range(8))
    assert h.group_device_ids([4, 2], ids, 0, 3) == [1, 3, 5, 7]
    assert h.group_device_ids([4, 2], ids, 1, 3) == [2, 3]
    assert h.group_device_ids([2, 2, 2], ids, 1, 5) == [5, 7]
    assert h.group_device_ids([8], ids, 0, 6) == ids
    assert h.group_device_ids([2, 2], [7, 5, 3, 1], 0, 1) == [5, 1]


def test_compute_local_shapes():
    assert h.compute_local_shapes([5, 9], [2], [0, 1], ["S1"]) == {0: [5, 5], 1: [5, 4]}
    assert h.compute_local_shapes([4, 8], [2], [0, 1], ["S0"]) == {0: [2, 8], 1: [2, 8]}
    even = h.compute_local_shapes([4, 16], [4, 2], list(range(8)), ["S0", "S1"])
    assert all(v == [1, 8] for v in even.values())
    # one tensor dim sharded by two mesh dims: row-major over them, uneven sizes by the shard rule
    merged = h.compute_local_shapes([4, 17], [4, 2], list(range(8)), ["S1", "S1"])
    assert merged == {0: [4, 3], **{i: [4, 2] for i in range(1, 8)}}
    p = h.compute_local_shapes([6, 5], [2], [0, 1], ["P"])
    assert p == {0: [6, 5], 1: [6, 5]}


@pytest.mark.parametrize("shape,mesh,ids,pl", [
    ([4, 8], [2], [0, 1], ["S2"]),      # shard dim beyond the rank
    ([1, 8], [2], [0, 1], ["S0"]),      # fewer rows than shards
    ([4, 8], [2], [0, 0], ["S0"]),      # duplicate device ids
    ([4, 8], [2], [0, 1], ["S0", "R"]),  # placements longer than the mesh
])
def test_check_valid_rejects(shape, mesh, ids, pl):
    with pytest.raises(Exception):
        h.check_valid(shape, mesh, ids, pl)


def test_check_valid_accepts():
    h.check_valid([5, 9], [2], [0, 1], ["S1"])
    h.check_valid([2, 16, 128, 128], [2, 2, 2], list(range(8)), ["S0", "S2", "S2"])


def test_sub_split_local_shapes():
    # piece i = shard-rule piece of the first s + 1 rows + shard-rule piece of the rest
    assert h.compute_local_shapes([6, 4], [2], [0, 1], ["S0/2"]) == {0: [4, 4], 1: [2, 4]}
    assert h.compute_local_shapes([9, 4], [2], [0, 1], ["S0/4"]) == {0: [5, 4], 1: [4, 4]}
    assert h.compute_local_shapes([2, 16, 3], [4], [0, 1, 2, 3], ["S1/7"]) == {i: [2, 4, 3] for i in range(4)}


def test_view_keeps_locals_and_checks_local_shapes():
    # Tensor.view(placements): metadata only; sub-split Shard(1, 4) of length 9 on 2 devices has local lengths
    # 5 and 4 (front 3+2, back 2+2), the same as Shard(1), so the view is allowed; Shard(0) is not
    torch = pytest.importorskip("torch")
    import dtorch_b200 as dtb
    mesh = dtb.DeviceMesh("cuda", [0, 1])
    locs = {0: torch.zeros(3, 5, 2), 1: torch.ones(3, 4, 2)}
    x = dtb.DTensor(locs, mesh, [dtb.Shard(1, 4)], (3, 9, 2))
    y = x.view([dtb.Shard(1)])
    assert y.placements == [dtb.Shard(1)] and y.local(1) is locs[1]
    assert y.view([dtb.Shard(1, 4)]).placements == [dtb.Shard(1, 4)]
    with pytest.raises(ValueError):
        x.view([dtb.Shard(0)])


def test_ring_overlap_argument_checks():
    torch = pytest.importorskip("torch")
    import dtorch_b200 as dtb
    mesh = dtb.DeviceMesh("cuda", [0, 1], mesh_dim_names=["ring"])
    t = dtb.DTensor({0: torch.zeros(1, 2, 4, 8), 1: torch.zeros(1, 2, 4, 8)}, mesh, [dtb.Shard(2)], (1, 2, 8, 8))
    for kw in ({"is_causal": True, "ring_cp_dim": "ring"}, {"dropout_p": 0.1, "ring_cp_dim": "ring"}, {}):
        with pytest.raises(ValueError):
            dtb.scaled_dot_product_attention_with_cp(t, t, t, ring_overlap=True, **kw)


def _local_shapes_restated(shape, mesh_shape, ids, placements):
    """DistributedSpec::ComputeLocalShape (dtorch/api/cpp/distributed_spec.cc:539-587) in plain Python: a tensor dim
    sharded by several mesh dims is split by the product of their sizes, row-major over those mesh dims, with the
    shard rule (the first L % k pieces one longer)."""
    import itertools
    info = {}
    for md, p in enumerate(placements):
        if p.startswith("S"):
            info.setdefault(int(p[1:]), []).append(md)
    out = {}
    for idx, coord in enumerate(itertools.product(*[range(m) for m in mesh_shape])):
        local = list(shape)
        for d, mds in info.items():
            k, sel = 1, 0
            for md in mds:
                k *= mesh_shape[md]
                sel = sel * mesh_shape[md] + coord[md]
            local[d] = shape[d] // k + (1 if sel < shape[d] % k else 0)
        out[ids[idx]] = local
    return out


def test_local_shapes_match_restatement_on_random_meshes():
    hyp = pytest.importorskip("hypothesis")
    st = pytest.importorskip("hypothesis.strategies")

    @hyp.settings(max_examples=300, deadline=None)
    @hyp.given(st.data())
    def check(data):
        mesh_shape = data.draw(st.lists(st.integers(2, 4), min_size=1, max_size=3))
        ndim = data.draw(st.integers(1, 4))
        placements = data.draw(st.lists(st.sampled_from(["R", "P"] + [f"S{d}" for d in range(ndim)]),
                                        min_size=len(mesh_shape), max_size=len(mesh_shape)))
        ways = {}
        for md, p in enumerate(placements):
            if p.startswith("S"):
                ways[int(p[1:])] = ways.get(int(p[1:]), 1) * mesh_shape[md]
        shape = [data.draw(st.integers(ways.get(d, 1), 3 * ways.get(d, 1) + 5)) for d in range(ndim)]
        count = 1
        for m in mesh_shape:
            count *= m
        ids = data.draw(st.permutations(list(range(count))))
        h.check_valid(shape, mesh_shape, ids, placements)
        got = h.compute_local_shapes(shape, mesh_shape, ids, placements)
        assert got == _local_shapes_restated(shape, mesh_shape, ids, placements)

    check()


def test_placements_from_dict():
    # python/dtorch/distributed_spec.py:233-305
    import dtorch_b200 as dtb
    mesh = dtb.init_device_mesh("cuda", (2, 2), mesh_dim_names=["dp", "cp"])
    S, R = dtb.Shard, dtb.Replicate
    assert dtb.get_placements_from_dict(mesh, {"dp": S(0), "cp": S(1)}) == [S(0), S(1)]
    assert dtb.get_placements_from_dict(mesh, {1: S(2)}, default_placement_mode="replicate") == [R(), S(2)]
    assert dtb.get_placements_from_dict(mesh, {"cp": S(2)}, [S(0), R()], "keep") == [S(0), S(2)]
    assert dtb.get_placements_from_dict(mesh, {}, default_placement_mode="replicate") == [R(), R()]
    with pytest.raises(KeyError):
        dtb.get_placements_from_dict(mesh, {"dp": S(0)})
    with pytest.raises(KeyError):
        dtb.get_placements_from_dict(mesh, {})
    with pytest.raises(TypeError):
        dtb.get_placements_from_dict(mesh, {"dp": S(0), 1: R()})
    with pytest.raises(ValueError):
        dtb.get_placements_from_dict(dtb.init_device_mesh("cuda", (2,)), {"dp": S(0)})
