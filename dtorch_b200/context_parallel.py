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


def scaled_dot_product_attention_with_cp(query: DTensor, key: DTensor, value: DTensor, dropout_p: float = 0.0,
                                         is_causal: bool = False, scale: Optional[float] = None,
                                         ulysses_cp_dim: Optional[Union[int, str]] = None,
                                         ring_cp_dim: Optional[Union[int, str]] = None,
                                         ring_overlap: bool = False) -> DTensor:
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
