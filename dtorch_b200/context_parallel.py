"""Context-parallel scaled-dot-product attention over DTensors (the reference's
python/dtorch/nn/scaled_dot_product_attention_with_cp.py:14-111, Ulysses and "ring" paths).

Layout (N, H, L, E); q, k and v are sharded on the sequence (Shard(2)) along the context-parallel mesh dims.

* Ulysses: the sequence-sharded q, k, v become head-sharded (Shard(2) -> Shard(1)) in ONE fused all-to-all
  launch per device (the reference issues three redistributes), each device runs attention for its heads over
  the whole sequence, and the output returns to Shard(2).
* "Ring" (as the reference implements it): K and V are all-gathered along the ring dim (Shard(2) ->
  Replicate) and each device attends its query chunk to the whole key/value sequence.

Without a causal mask the order of the sequence does not matter, so sub-split sequence shards are viewed as
plain Shard(2) for the call and the output is viewed back (scaled_dot_product_attention_with_cp.py:44-62,
:111-112). With `is_causal` each device calls torch's attention on its local query chunk with `is_causal=True`,
as the reference's SdpaOp::Compute does (scaled_dot_product_attention_op.cc:104-109): for a local query chunk
shorter than the gathered key sequence that is torch's top-left aligned mask.

`ulysses_overlap_groups=G` (batch 1, one q/k/v shape) pipelines the Ulysses path over G head groups: the
executor runs each group's q/k/v swap and swap back on its kernel streams without making the caller's streams
wait, and each device's attention of group g waits only for group g's swap, so swaps of neighbouring groups run
while group g attends. Results equal the plain path's bit for bit.

`ring_overlap=True` (non-causal, no dropout) overlaps the K/V all-gather with attention: each device attends
its query chunk to its own key/value chunk on a side stream while the all-gather runs, then to the other
devices' chunks, and merges the partial outputs by their log-sum-exp (softmax over the union of the chunks).
The result equals the one-pass attention up to floating-point rounding. It is off by default: on B200 the
split (attention kernels that also return the log-sum-exp, the fp32 merge, more launches) cost more than the
all-gather it hides at every shape measured (2 GPUs, bf16, sequence 1K-16K, 16-64 heads).
"""

from __future__ import annotations

from typing import Dict, Optional, Union

import torch
import torch.nn.functional as F

from .dtensor import DTensor, Replicate, Shard, _host, redistribute_many


def _dim_index(tensor: DTensor, dim: Optional[Union[int, str]]) -> Optional[int]:
    if dim is None:
        return None
    if isinstance(dim, str):
        if dim not in tensor.device_mesh.dim_names:
            return None
        dim = tensor.device_mesh.dim_names.index(dim)
    return None if tensor.device_mesh.shape[dim] == 1 else dim


def _attend_with_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float]):
    """Attention of q to one key/value chunk, and the log-sum-exp of each query row's scaled scores
    (fp32, (N, H, L))."""
    if q.dtype in (torch.float16, torch.bfloat16) and q.shape[-1] % 8 == 0 and q.shape[-1] <= 128:
        # cuDNN's fused attention: the kernel torch's own dispatch picks for these inputs on B200
        out, lse = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, v, None, True, 0.0, False, False,
                                                                      scale=scale)[:2]
        return out, lse.reshape(lse.shape[:3])
    # the memory-efficient kernel (its log-sum-exp rows are padded to a multiple of 32)
    out, lse = torch.ops.aten._scaled_dot_product_efficient_attention(q, k, v, None, True, 0.0, False, scale=scale)[:2]
    return out, lse[..., : q.shape[2]]


def _merge_partials(parts, dtype) -> torch.Tensor:
    """Softmax attention over the union of key chunks from per-chunk outputs o_i and log-sum-exps l_i:
    l = logsumexp_i l_i, o = sum_i exp(l_i - l) o_i (in fp32)."""
    lse = torch.logsumexp(torch.stack([l for _, l in parts]), dim=0)
    acc = None
    for o, l in parts:
        term = torch.exp(l - lse).unsqueeze(-1) * o.float()
        acc = term if acc is None else acc + term
    return acc.to(dtype)


def _ring_attention_overlapped(query: DTensor, key: DTensor, value: DTensor, r: int,
                               scale: Optional[float]) -> Dict[int, torch.Tensor]:
    mesh = query.device_mesh
    own, side = {}, {}
    for gid in mesh.ids:
        q, k, v = query.local(gid), key.local(gid), value.local(gid)
        with torch.cuda.device(q.device):
            s = torch.cuda.Stream(q.device)
            s.wait_stream(torch.cuda.current_stream(q.device))
            with torch.cuda.stream(s):
                own[gid] = _attend_with_lse(q, k, v, scale)
            for t in (q, k, v):
                t.record_stream(s)
            side[gid] = s
    kv = list(query.placements)
    kv[r] = Replicate()
    key_full, value_full = redistribute_many([key, value], kv)
    out = {}
    for gid in mesh.ids:
        q, kf, vf = query.local(gid), key_full.local(gid), value_full.local(gid)
        group = _host.group_device_ids(list(mesh.shape), mesh.ids, r, gid)
        rank = group.index(gid)
        off = sum(key.local(g).shape[2] for g in group[:rank])
        end = off + key.local(gid).shape[2]
        with torch.cuda.device(q.device):
            cur = torch.cuda.current_stream(q.device)
            parts = []
            if off > 0:
                parts.append(_attend_with_lse(q, kf[:, :, :off], vf[:, :, :off], scale))
            if end < kf.shape[2]:
                parts.append(_attend_with_lse(q, kf[:, :, end:], vf[:, :, end:], scale))
            cur.wait_stream(side[gid])
            for t in own[gid]:
                t.record_stream(cur)
            parts.append(own[gid])
            out[gid] = _merge_partials(parts, q.dtype)
    return out


class _KernelStreams:
    """The executor's kernel stream of every device, and events that mark how far a collective enqueued there
    has got."""

    def __init__(self, ids):
        self.streams = {}
        for gid in ids:
            ptr, dev = _host.kernel_stream(gid)
            self.streams[gid] = torch.cuda.ExternalStream(ptr, device=torch.device("cuda", dev))

    def mark(self):
        evs = {}
        for gid, s in self.streams.items():
            e = torch.cuda.Event()
            e.record(s)
            evs[gid] = e
        return evs


def _ulysses_overlapped(query: DTensor, key: DTensor, value: DTensor, u: int, groups: int, dropout_p: float,
                        is_causal: bool, scale: Optional[float]) -> DTensor:
    """Ulysses attention pipelined over `groups` head groups. The executor runs the collectives on its kernel
    streams without making the caller's streams wait (deferred hand-off); the caller's stream of each device
    waits for a group's q/k/v swap only right before that group's attention. So the swap of group g + 1 and the
    swap back of group g - 1 run while group g attends. Each group's heads split over the ranks as in the plain
    path and attention is independent per head: the result equals the plain path's bit for bit."""
    mesh = query.device_mesh
    seq = list(query.placements)
    head = list(seq)
    head[u] = Shard(1)
    H, hg = query.shape[1], query.shape[1] // groups
    ks = _KernelStreams(mesh.ids)
    mesh_shape, ids = list(mesh.shape), mesh.ids
    src_p, head_p = [repr(p) for p in seq], [repr(p) for p in head]

    def swap(g):
        lo, hi = g * hg, (g + 1) * hg
        parts = [{gid: t.local(gid)[:, lo:hi] for gid in ids} for t in (query, key, value)]
        shape = [query.shape[0], hg] + list(query.shape[2:])
        outs = _host.redistribute_multi(parts, mesh_shape, ids, src_p, head_p, shape, handoff=False)
        return outs, ks.mark()

    pending = swap(0)
    backs = []
    for g in range(groups):
        nxt = swap(g + 1) if g + 1 < groups else None  # enqueued before this group's attention
        (qs, kk, vs), ready = pending
        att = {}
        for gid in ids:
            dev = qs[gid].device
            with torch.cuda.device(dev):
                cur = torch.cuda.current_stream(dev)
                cur.wait_event(ready[gid])
                for t in (qs[gid], kk[gid], vs[gid]):
                    t.record_stream(cur)
                att[gid] = F.scaled_dot_product_attention(qs[gid], kk[gid], vs[gid], dropout_p=dropout_p,
                                                          is_causal=is_causal, scale=scale)
        shape = [query.shape[0], hg, query.shape[2], value.shape[3]]
        back = _host.redistribute(att, mesh_shape, ids, head_p, src_p, shape, handoff=False)
        backs.append((back, ks.mark()))
        pending = nxt
    # every group's output back in sequence-sharded layout, concatenated along the heads on the caller's stream
    out_locals = {}
    for gid in ids:
        dev = query.local(gid).device
        with torch.cuda.device(dev):
            cur = torch.cuda.current_stream(dev)
            pieces = []
            for back, done in backs:
                cur.wait_event(done[gid])
                back[gid].record_stream(cur)
                pieces.append(back[gid])
            out_locals[gid] = torch.cat(pieces, dim=1)
    return DTensor(out_locals, mesh, seq, tuple(query.shape[:3]) + (value.shape[3],))


def scaled_dot_product_attention_with_cp(query: DTensor, key: DTensor, value: DTensor, dropout_p: float = 0.0,
                                         is_causal: bool = False, scale: Optional[float] = None,
                                         ulysses_cp_dim: Optional[Union[int, str]] = None,
                                         ring_cp_dim: Optional[Union[int, str]] = None,
                                         ring_overlap: bool = False, ulysses_overlap_groups: int = 1) -> DTensor:
    """`ulysses_overlap_groups` > 1 pipelines a pure-Ulysses call over that many head groups (batch 1, q/k/v of
    one shape, heads divisible by groups * Ulysses size): swaps of one group overlap attention of another."""
    u = _dim_index(query, ulysses_cp_dim)
    r = _dim_index(query, ring_cp_dim)
    if ring_overlap and (r is None or is_causal or dropout_p > 0.0):
        raise ValueError("ring_overlap needs a ring dim, is_causal=False and dropout_p=0")
    if key.placements != query.placements or value.placements != query.placements:
        raise RuntimeError("query, key and value have different placements")
    old_placements = list(query.placements)
    if not is_causal:
        plain = [Shard(p.get_shard_index()) if p.is_shard() and p.has_sub_split_coordinates() else p
                 for p in old_placements]
        query, key, value = query.view(plain), key.view(plain), value.view(plain)
    for d in (u, r):
        if d is not None and query.placements[d] != Shard(2):
            raise ValueError("context-parallel dims must shard the sequence dim (Shard(2))")
    mesh = query.device_mesh
    placements = list(query.placements)
    if u is not None and r is None and ulysses_overlap_groups > 1:
        n = mesh.shape[u]
        if not (query.shape == key.shape == value.shape and query.shape[0] == 1
                and query.shape[1] % (ulysses_overlap_groups * n) == 0):
            raise ValueError("ulysses_overlap_groups needs q, k, v of one shape, batch 1 and heads divisible by "
                             "groups x Ulysses size")
        out = _ulysses_overlapped(query, key, value, u, ulysses_overlap_groups, dropout_p, is_causal, scale)
        return out if is_causal else out.view(old_placements)
    if u is not None:
        n = mesh.shape[u]
        if query.shape[1] % n or key.shape[1] % n:
            raise ValueError(f"attention heads ({query.shape[1]}, {key.shape[1]}) cannot be divided evenly by the "
                             f"Ulysses size {n}")
        head = list(placements)
        head[u] = Shard(1)
        if query.shape == key.shape == value.shape:
            query, key, value = redistribute_many([query, key, value], head)
        else:
            query = query.redistribute(placements=head)
            key, value = redistribute_many([key, value], head)
    if ring_overlap:
        out_locals = _ring_attention_overlapped(query, key, value, r, scale)
    else:
        if r is not None:
            kv = list(query.placements)
            kv[r] = Replicate()
            key, value = redistribute_many([key, value], kv)
        out_locals = {}
        for gid in mesh.ids:
            q, k, v = query.local(gid), key.local(gid), value.local(gid)
            with torch.cuda.device(q.device):
                out_locals[gid] = F.scaled_dot_product_attention(q, k, v, dropout_p=dropout_p, is_causal=is_causal,
                                                                 scale=scale)
    out_shape = tuple(query.shape[:3]) + (value.shape[3],)
    out = DTensor(out_locals, mesh, query.placements, out_shape)
    if u is not None:
        out = out.redistribute(placements=placements)
    return out if is_causal else out.view(old_placements)
