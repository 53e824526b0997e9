"""DeviceMesh / Placement / DTensor.redistribute over the B200 collectives.

The user-facing names and argument meaning follow the reference's Python API (python/dtorch/distributed_spec.py:
``DeviceMesh``, ``Shard``, ``Replicate``, ``Partial``, ``init_device_mesh``; python/dtorch/tensor.py:299-351:
``Tensor.redistribute``, ``redistribute_like``). A DTensor here is the set of its per-device local tensors;
``redistribute`` runs the C++ executor (one kernel-stream thread per device, one ThreadGroup collective per
changed mesh dim, ``dtorch_b200/csrc/host/redistribute.cpp``). ``from_torch`` / ``to_torch`` place and collect
a whole tensor the way the reference's DistributedScather / DistributeGather do
(dtorch/core/kernel/kernel_implement/distributed_scather_and_gather.cc:24-145); they are host-side helpers,
not part of the collective path.
"""

from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Sequence, Union

import torch

from . import _host


class Placement:
    """Replicate ("R"), Partial ("P", pending SUM), Shard(dim) ("S<dim>") or the sub-split Shard(dim, s)
    ("S<dim>/<s>": rank i holds piece i of the first s + 1 rows plus piece i of the rest -- the causal
    load-balancing layout of the reference's context parallelism)."""

    def __init__(self, placement: str):
        self._s = placement
        self._sub = -1
        if placement in ("R", "P"):
            self._dim = None
        elif placement.startswith("S"):
            body = placement[1:]
            if "/" in body:
                body, sub = body.split("/")
                self._sub = int(sub)
            self._dim = int(body)
        else:
            raise ValueError(f"bad placement {placement!r}")

    def has_sub_split_coordinates(self) -> bool:
        return self._sub != -1

    def get_sub_split_coordinates(self) -> int:
        return self._sub

    def __eq__(self, other) -> bool:
        return isinstance(other, Placement) and other._s == self._s

    def __hash__(self):
        return hash(self._s)

    def __repr__(self) -> str:
        return self._s

    def is_replicate(self) -> bool:
        return self._s == "R"

    def is_partial(self) -> bool:
        return self._s == "P"

    def is_shard(self) -> bool:
        return self._dim is not None

    def get_shard_index(self) -> int:
        return self._dim


def Shard(dim: int, sub_split_coordinates: int = -1) -> Placement:  # noqa: N802 (reference API name)
    return Placement(f"S{dim}" if sub_split_coordinates == -1 else f"S{dim}/{sub_split_coordinates}")


def Replicate() -> Placement:  # noqa: N802
    return Placement("R")


def Partial() -> Placement:  # noqa: N802
    return Placement("P")


class DeviceMesh:
    """Global device ids arranged in a mesh. Only "cuda" meshes are served by this library; the reference's
    CPU mesh is its own thread-group path (the test oracle), not a fallback."""

    def __init__(self, device_type: str, mesh, mesh_dim_names: Optional[Sequence[str]] = None):
        if device_type not in ("cuda", "gpu"):
            raise ValueError("dtorch_b200 serves cuda device meshes only")
        t = mesh if isinstance(mesh, torch.Tensor) else torch.tensor(mesh)
        t = t.cpu().to(torch.int64)
        if t.dim() == 0:
            t = t.reshape(1)
        self.mesh = t
        self.device_type = "cuda"
        self.dim_names = list(mesh_dim_names) if mesh_dim_names else []
        # the mesh is immutable: its shape and ids are read on every redistribute, so keep them at hand
        self._shape = tuple(int(x) for x in t.shape)
        self._ids = [int(x) for x in t.reshape(-1).tolist()]

    @property
    def shape(self):
        return self._shape

    @property
    def ndim(self) -> int:
        return len(self._shape)

    @property
    def ids(self) -> List[int]:
        return list(self._ids)

    @property
    def is_distributed(self) -> bool:
        return self.mesh.numel() > 1

    def has_dim_name(self, dim_name: str) -> bool:
        return dim_name in self.dim_names

    def dim_name_index(self, dim_name: str, default_value: Optional[int] = None) -> Optional[int]:
        return self.dim_names.index(dim_name) if dim_name in self.dim_names else default_value

    def __eq__(self, other) -> bool:
        return isinstance(other, DeviceMesh) and self._shape == other._shape and self._ids == other._ids

    def __repr__(self) -> str:
        return f"DeviceMesh('cuda', shape: {self.shape}, data: {self.mesh.tolist()})"


def init_device_mesh(device_type: str, mesh_shape: Union[int, Sequence[int]],
                     mesh_dim_names: Optional[Sequence[str]] = None) -> DeviceMesh:
    """Mesh of devices 0..prod(shape)-1 in row-major order (python/dtorch/distributed_spec.py:179-194)."""
    if isinstance(mesh_shape, int):
        mesh_shape = (mesh_shape,)
    mesh_shape = [s for s in mesh_shape if s is not None] or [1]
    return DeviceMesh(device_type, torch.arange(math.prod(mesh_shape)).view(mesh_shape), mesh_dim_names)


def get_placements_from_dict(device_mesh: DeviceMesh, placements_dict: Dict[Union[str, int], Placement],
                             original_placements: Optional[Sequence[Placement]] = None,
                             default_placement_mode: str = "raise_error") -> List[Placement]:
    """Placements per mesh dim from a dict keyed by mesh dim name or index (python/dtorch/distributed_spec.py:
    233-305). Dims the dict does not name get Replicate ("replicate"), keep their current placement ("keep"),
    or raise KeyError ("raise_error")."""
    if default_placement_mode not in ("raise_error", "replicate", "keep"):
        raise ValueError(f"unknown default_placement_mode {default_placement_mode!r}")
    if device_mesh.ndim == 0:
        return []
    if default_placement_mode == "keep" and (original_placements is None
                                            or len(original_placements) != device_mesh.ndim):
        raise ValueError("default_placement_mode='keep' needs one original placement per mesh dim")
    if not placements_dict:
        if default_placement_mode == "replicate":
            return [Replicate()] * device_mesh.ndim
        if default_placement_mode == "keep":
            return list(original_placements)
        raise KeyError("placements_dict is empty and default_placement_mode is 'raise_error'")
    by_name = all(isinstance(k, str) for k in placements_dict)
    if not by_name and not all(isinstance(k, int) for k in placements_dict):
        raise TypeError("placements_dict keys must be all mesh dim names or all mesh dim indices")
    if by_name and len(device_mesh.dim_names) != device_mesh.ndim:
        raise ValueError("placements_dict is keyed by dim name but the device mesh has no dim names")
    out = []
    for i in range(device_mesh.ndim):
        key = device_mesh.dim_names[i] if by_name else i
        if key in placements_dict:
            out.append(placements_dict[key])
        elif default_placement_mode == "replicate":
            out.append(Replicate())
        elif default_placement_mode == "keep":
            out.append(original_placements[i])
        else:
            raise KeyError(f"mesh dim {key!r} is not in placements_dict {placements_dict}")
    return out


def cuda_device_of(global_id: int) -> int:
    """CUDA ordinal of a global device id (all on device 0 when DTORCH_DTENSOR_IN_SAME_DEVICE=1)."""
    return 0 if os.environ.get("DTORCH_DTENSOR_IN_SAME_DEVICE") == "1" else int(global_id)


def _strings(placements: Sequence[Placement]) -> List[str]:
    return [repr(p) for p in placements]


def _merge_same_shard_dims(mesh: torch.Tensor, placements: List[Placement]):
    """Merge mesh dims sharding the same tensor dim into one (DistributedSpec::MergeSameShardDim,
    distributed_spec.cc:442-489), so a tensor dim sharded over several mesh dims splits row-major."""
    groups: Dict[int, List[int]] = {}
    for i, p in enumerate(placements):
        if p.is_shard():
            groups.setdefault(p.get_shard_index(), []).append(i)
    merge = {g[0]: g for g in groups.values() if len(g) > 1}
    if not merge:
        return mesh, placements
    perm, new_shape, new_p, used = [], [], [], set()
    for i in range(mesh.dim()):
        if i in used:
            continue
        dims = merge.get(i, [i])
        for d in dims:
            perm.append(d)
            used.add(d)
        new_shape.append(math.prod(mesh.shape[d] for d in dims))
        new_p.append(placements[i])
    return mesh.permute(perm).reshape(new_shape), new_p


def _to_device(t: torch.Tensor, device: int) -> torch.Tensor:
    """`t` on CUDA device `device`: itself when it is there already, else a new tensor filled by dt_peer_copy (a
    kernel on t's GPU storing into the destination over NVLink), ordered after the current streams of both
    devices and before later work on the destination's current stream."""
    if t.device.type != "cuda":
        return t.to(f"cuda:{device}")
    if t.device.index == device:
        return t
    from . import capi

    t = t.contiguous()
    src = t.device.index
    out = torch.empty(t.shape, dtype=t.dtype, device=f"cuda:{device}")
    s_src, s_dst = torch.cuda.current_stream(src), torch.cuda.current_stream(device)
    s_src.wait_stream(s_dst)  # the destination buffer is free once the destination's stream got here
    capi.peer_copy(out.data_ptr(), device, t.data_ptr(), src, t.numel() * t.element_size(), s_src.cuda_stream)
    s_dst.wait_stream(s_src)
    out.record_stream(s_src)
    return out


def set_pool_bytes(nbytes: int) -> None:
    """Give every device group created from now on a symmetric pool of `nbytes` per GPU (0: none; the default
    comes from DTORCH_B200_POOL_MB). DTensor locals placed by ``from_torch`` / ``empty`` on a 1-D mesh and the
    outputs of every collective then sit at the same offset on every GPU of the group, so collectives on them
    need no pointer exchange; where the GPUs support NVLink multicast the pool is the group's NVLS buffer and
    all-reduces on it reduce inside the NVSwitch (fp32 accumulation, the switch's order: within the reductions'
    tolerance rather than bit-identical to the rank-order fold). Call before the group's first collective."""
    _host.set_pool_bytes(int(nbytes))


def _pool_group(device_mesh: DeviceMesh) -> Optional[List[int]]:
    """The device group whose pool holds the locals of a DTensor on `device_mesh` (1-D peer meshes only)."""
    if device_mesh.ndim != 1 or len(device_mesh.ids) < 2 or _host.pool_bytes() == 0:
        return None
    if os.environ.get("DTORCH_DTENSOR_IN_SAME_DEVICE") == "1":
        return None
    return device_mesh.ids


def _place_locals(parts: Dict[int, torch.Tensor], device_mesh: DeviceMesh) -> Dict[int, torch.Tensor]:
    """Each device's part on its GPU: in the group's symmetric pool when it has one (one block per device,
    sized for the largest part, in mesh order on every device), else an ordinary allocation."""
    group = _pool_group(device_mesh)
    out: Dict[int, torch.Tensor] = {}
    if group is not None:
        nbytes = max(t.numel() * t.element_size() for t in parts.values())
        for gid in group:
            t = parts[gid]
            dst = _host.pool_empty(group, gid, list(t.shape), t.dtype, nbytes)
            dst.copy_(t)
            out[gid] = dst
        return out
    for gid, t in parts.items():
        out[gid] = t.contiguous().to(f"cuda:{cuda_device_of(gid)}")
    return out


class DTensor:
    """A distributed tensor: one local tensor per global device id of `device_mesh`."""

    def __init__(self, locals_: Dict[int, torch.Tensor], device_mesh: DeviceMesh, placements: Sequence[Placement],
                 shape: Sequence[int]):
        self._locals = dict(locals_)
        self.device_mesh = device_mesh
        self.placements = list(placements)
        self.shape = tuple(int(s) for s in shape)

    @property
    def dtype(self):
        return next(iter(self._locals.values())).dtype

    def local(self, device_id: int) -> torch.Tensor:
        return self._locals[device_id]

    @property
    def locals(self) -> Dict[int, torch.Tensor]:
        return dict(self._locals)

    @staticmethod
    def empty(shapes: Dict[int, Sequence[int]], dtype, device_mesh: DeviceMesh, placements: Sequence[Placement],
              shape: Sequence[int]) -> "DTensor":
        """A DTensor of uninitialised locals with the given per-device shapes, allocated like ``from_torch``'s
        (in the group's symmetric pool when it has one)."""
        group = _pool_group(device_mesh)
        es = torch.tensor([], dtype=dtype).element_size()
        out: Dict[int, torch.Tensor] = {}
        if group is not None:
            nbytes = max(math.prod(s) * es for s in shapes.values())
            for gid in group:
                out[gid] = _host.pool_empty(group, gid, list(shapes[gid]), dtype, nbytes)
        else:
            for gid in device_mesh.ids:
                out[gid] = torch.empty(list(shapes[gid]), dtype=dtype, device=f"cuda:{cuda_device_of(gid)}")
        return DTensor(out, device_mesh, placements, shape)

    # -- placement of a whole tensor (host helpers) -------------------------------------------------------
    @staticmethod
    def from_torch(tensor: torch.Tensor, device_mesh: DeviceMesh, placements: Sequence[Placement]) -> "DTensor":
        placements = _host.normalize(_strings(placements), list(device_mesh.shape), device_mesh.ids, tensor.dim())
        placements = [Placement(p) for p in placements]
        _host.check_valid(list(tensor.shape), list(device_mesh.shape), device_mesh.ids, _strings(placements))
        mesh, plc = _merge_same_shard_dims(device_mesh.mesh, placements)
        parts_of: Dict[int, torch.Tensor] = {}

        def scatter(t: torch.Tensor, m: torch.Tensor, i: int):
            if i == len(plc):
                parts_of[int(m.reshape(-1)[0])] = t
                return
            n = m.shape[0]
            p = plc[i]
            if p.is_replicate():
                parts = [t] * n
            elif p.is_shard() and p.has_sub_split_coordinates():
                d, sub = p.get_shard_index(), p.get_sub_split_coordinates()
                front, back = torch.split(t, [sub + 1, t.shape[d] - sub - 1], d)
                fronts = torch.split(front, _host.shard_sizes(sub + 1, n), d)
                backs = torch.split(back, _host.shard_sizes(t.shape[d] - sub - 1, n), d)
                parts = [torch.cat([fronts[k], backs[k]], d) for k in range(n)]
            elif p.is_shard():
                d = p.get_shard_index()
                parts = list(torch.split(t, _host.shard_sizes(t.shape[d], n), d))
            else:  # Partial: the tensor on the first, zeros elsewhere (distributed_scather_and_gather.cc:83-84)
                parts = [t] + [torch.zeros_like(t)] * (n - 1)
            for k in range(n):
                scatter(parts[k], m[k], i + 1)

        scatter(tensor, mesh, 0)
        return DTensor(_place_locals(parts_of, device_mesh), device_mesh, placements, tensor.shape)

    def to_torch(self, device: Union[str, torch.device] = "cpu") -> torch.Tensor:
        mesh, plc = _merge_same_shard_dims(self.device_mesh.mesh, self.placements)

        dev = torch.device(device)

        def gather(m: torch.Tensor, i: int) -> torch.Tensor:
            if i == len(plc):
                t = self._locals[int(m.reshape(-1)[0])]
                return _to_device(t, dev.index if dev.index is not None else torch.cuda.current_device()) \
                    if dev.type == "cuda" else t.to(dev)
            p = plc[i]
            if p.is_replicate():
                return gather(m[0], i + 1)
            parts = [gather(m[k], i + 1) for k in range(m.shape[0])]
            if p.is_shard() and p.has_sub_split_coordinates():
                d, sub = p.get_shard_index(), p.get_sub_split_coordinates()
                fs = _host.shard_sizes(sub + 1, len(parts))
                fronts = [x.narrow(d, 0, fs[k]) for k, x in enumerate(parts)]
                backs = [x.narrow(d, fs[k], x.shape[d] - fs[k]) for k, x in enumerate(parts)]
                return torch.cat([torch.cat(fronts, d), torch.cat(backs, d)], d)
            if p.is_shard():
                return torch.cat(parts, p.get_shard_index())
            acc = parts[0]
            for x in parts[1:]:
                acc = acc + x
            return acc

        return gather(mesh, 0)

    # -- redistribute (the hot path) -----------------------------------------------------------------------
    def redistribute(self, device_mesh: Optional[DeviceMesh] = None,
                     placements: Optional[Sequence[Placement]] = None) -> "DTensor":
        """Tensor.redistribute (python/dtorch/tensor.py:299-309): same mesh, new placements."""
        assert device_mesh is not None or placements is not None
        device_mesh = device_mesh if device_mesh is not None else self.device_mesh
        placements = list(placements) if placements is not None else list(self.placements)
        if device_mesh != self.device_mesh:
            # placements first on the current mesh, then the move (ConvertKernel::ConvertDeviceMesh,
            # convert_kernel.cc:79-102: rank i of the source mesh hands its local tensor to rank i of the
            # destination mesh)
            here = self.redistribute(placements=placements) if placements != self.placements else self
            return here._move_to_mesh(device_mesh)
        new = _host.redistribute(self._locals, list(device_mesh.shape), device_mesh.ids, _strings(self.placements),
                                 _strings(placements), list(self.shape))
        normalized = _host.normalize(_strings(placements), list(device_mesh.shape), device_mesh.ids, len(self.shape))
        return DTensor(new, device_mesh, [Placement(p) for p in normalized], self.shape)

    def _move_to_mesh(self, mesh: DeviceMesh) -> "DTensor":
        if tuple(mesh.shape) != tuple(self.device_mesh.shape):
            raise ValueError(f"device meshes differ in shape: {self.device_mesh.shape} vs {mesh.shape}")
        out = {}
        for src, dst in zip(self.device_mesh.ids, mesh.ids):
            # rank i of the source mesh hands its local to rank i of the destination mesh: a kernel on the
            # source GPU stores it straight into the destination GPU's memory over NVLink
            out[dst] = _to_device(self._locals[src], cuda_device_of(dst))
        return DTensor(out, mesh, self.placements, self.shape)

    def redistribute_like(self, other: "DTensor") -> "DTensor":
        return self.redistribute(device_mesh=other.device_mesh, placements=other.placements)

    def redistribute_by_dict(self, device_mesh: Optional[DeviceMesh] = None,
                             placements_dict: Optional[Dict[Union[str, int], Placement]] = None, *,
                             default_placement_mode: str = "raise_error",
                             convert_shard_size_one_to_replicate: bool = True) -> "DTensor":
        """Tensor.redistribute_by_dict (python/dtorch/tensor.py:317-351): placements named per mesh dim; a
        Shard of a tensor dim of size 1 becomes Replicate unless told otherwise."""
        device_mesh = device_mesh if device_mesh is not None else self.device_mesh
        if placements_dict:
            if device_mesh.is_distributed:
                placements = get_placements_from_dict(device_mesh, placements_dict, self.placements,
                                                      default_placement_mode)
            else:
                placements = [Replicate()] * device_mesh.ndim
        else:
            placements = list(self.placements)
        if convert_shard_size_one_to_replicate:
            placements = [Replicate() if p.is_shard() and self.shape[p.get_shard_index()] == 1 else p
                          for p in placements]
        return self.redistribute(device_mesh=device_mesh, placements=placements)

    def view(self, placements: Sequence[Placement]) -> "DTensor":
        """Tensor.view(placements) (python/dtorch/tensor.py:439-447): the same local tensors read under other
        placements, no data movement (e.g. Shard(2, s) viewed as Shard(2) when the order of the sequence does
        not matter). Every device's local shape must stay the same."""
        mesh = self.device_mesh
        placements = [Placement(p) for p in _host.normalize(_strings(placements), list(mesh.shape), mesh.ids,
                                                            len(self.shape))]
        _host.check_valid(list(self.shape), list(mesh.shape), mesh.ids, _strings(placements))
        shapes = _host.compute_local_shapes(list(self.shape), list(mesh.shape), mesh.ids, _strings(placements))
        for gid, t in self._locals.items():
            if list(t.shape) != list(shapes[gid]):
                raise ValueError(f"view {placements} changes device {gid}'s local shape {tuple(t.shape)} to "
                                 f"{tuple(shapes[gid])}")
        return DTensor(self._locals, mesh, placements, self.shape)

    def __repr__(self) -> str:
        return f"DTensor(shape={self.shape}, mesh={self.device_mesh}, placements={self.placements})"


def clear() -> None:
    """Destroy the kernel-stream threads and communicators (e.g. before switching device-mapping modes)."""
    _host.clear()


def redistribute_many(tensors: Sequence[DTensor], placements: Sequence[Placement]) -> List[DTensor]:
    """Redistribute DTensors of one shape, mesh and placement to the same new placements. When the change is
    Shard(i) -> Shard(j) on one mesh dim, all of them move in one fused all-to-all launch per device."""
    first = tensors[0]
    for t in tensors[1:]:
        if t.shape != first.shape or t.placements != first.placements or t.device_mesh != first.device_mesh:
            raise ValueError("redistribute_many: tensors differ in shape, placements or mesh")
    mesh = first.device_mesh
    outs = _host.redistribute_multi([t._locals for t in tensors], list(mesh.shape), mesh.ids,
                                    _strings(first.placements), _strings(placements), list(first.shape))
    normalized = _host.normalize(_strings(placements), list(mesh.shape), mesh.ids, len(first.shape))
    return [DTensor(o, mesh, [Placement(p) for p in normalized], first.shape) for o in outs]


def reduce(tensor: DTensor, dims: Union[int, Sequence[int]], kind: str = "sum", keepdim: bool = False) -> DTensor:
    """Sum or mean over tensor dims of a DTensor (the reference's ReduceKernel::Compute,
    dtorch/core/kernel/kernel_implement/reduce_kernel.cc:63-116). Each device reduces its shard; a mesh dim that
    sharded a reduced dim leaves the result Partial, and one all-reduce per such mesh dim (rank-order fp32 fold)
    makes it Replicate -- instead of the reference's all-gather of every rank's partial and a host-side fold,
    which moves n times the data. `mean` divides the global sum by the global element count (for uneven shards
    the reference's mean of per-rank means is not the mean)."""
    if kind not in ("sum", "mean"):
        raise ValueError("kind must be 'sum' or 'mean'")
    nd = len(tensor.shape)
    dims = [dims] if isinstance(dims, int) else list(dims)
    dims = sorted({d % nd for d in dims})
    if any(p.is_partial() for p in tensor.placements):
        raise ValueError("reduce of a Partial DTensor: redistribute it first")
    locals_ = {gid: t.sum(dim=dims, keepdim=keepdim) for gid, t in tensor._locals.items()}
    placements, to_replicate = [], []
    for p in tensor.placements:
        if p.is_shard() and p.get_shard_index() in dims:
            placements.append(Partial())
            to_replicate.append(Replicate())
        elif p.is_shard() and not keepdim:
            d = p.get_shard_index()
            placements.append(Shard(d - sum(1 for r in dims if r < d)))
            to_replicate.append(placements[-1])
        else:
            placements.append(p)
            to_replicate.append(p)
    shape = [1 if i in dims else s for i, s in enumerate(tensor.shape)] if keepdim else \
        [s for i, s in enumerate(tensor.shape) if i not in dims]
    out = DTensor(locals_, tensor.device_mesh, placements, shape)
    if placements != to_replicate:
        out = out.redistribute(placements=to_replicate)
    if kind == "mean":
        count = math.prod(tensor.shape[d] for d in dims)
        out = DTensor({g: t / count for g, t in out._locals.items()}, out.device_mesh, out.placements, out.shape)
    return out
