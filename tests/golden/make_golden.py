"""Generate tests/golden/*.npz: seeded inputs and the outputs of the reference's OWN thread-group code.

Outputs come from oracle/_ref/libdtref.so -- the reference's ThreadGroup, ThreadGroupSameDeviceBackend and
MemoryTensorStore sources compiled out of tree (oracle/Makefile, target ``ref``) and run on a CPU DeviceMesh
by n rank threads. Regenerate with ``python tests/golden/make_golden.py`` where the reference sources exist.

Each case stores ``in_<r>`` (raw storage, uint16 bits for bf16/fp16), ``out_<r>`` and a JSON ``meta``.
"""

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.oracle import Reference, shard_sizes  # noqa: E402

DT = {"float32": (torch.float32, 0), "bfloat16": (torch.bfloat16, 1), "float16": (torch.float16, 2)}


def raw(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().numpy().copy()
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def gen(shape, dtype, seed, dist):
    g = torch.Generator().manual_seed(seed)
    if dist == "rand":
        t = torch.rand(*shape, generator=g)
    elif dist == "uniform":
        t = torch.rand(*shape, generator=g) * 2 - 1
    else:
        t = torch.randn(*shape, generator=g)
    return t.to(DT[dtype][0])


def save(name, ins, outs, meta):
    arrs = {f"in_{r}": a for r, a in enumerate(ins)}
    arrs.update({f"out_{r}": a for r, a in enumerate(outs)})
    arrs["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)


def main():
    ref = Reference()
    cases = 0
    # Partial -> Replicate / Partial -> Shard(0): rank r's partial from seed + r
    for n, dtype, count, dist in [(2, "float32", 1000, "rand"), (4, "float32", 4099, "randn"),
                                  (8, "float32", 2048, "uniform"), (2, "bfloat16", 777, "randn"),
                                  (4, "bfloat16", 4096, "randn"), (8, "bfloat16", 8200, "randn"),
                                  (3, "float16", 1001, "randn"), (8, "float16", 1024, "uniform")]:
        ins = [raw(gen((count,), dtype, 100 + r, dist)) for r in range(n)]
        outs, _ = ref.all_reduce(ins, DT[dtype][1])
        save(f"all_reduce_n{n}_{dtype}_{count}", ins, outs, {"op": "all_reduce", "n": n, "dtype": dtype})
        cases += 1
    for n, dtype, rows, cols, dist in [(2, "float32", 8, 5, "rand"), (4, "bfloat16", 16, 33, "randn"),
                                       (8, "float32", 64, 17, "randn"), (8, "bfloat16", 16, 64, "randn"),
                                       (3, "float16", 9, 7, "randn")]:
        ins = [raw(gen((rows * cols,), dtype, 200 + r, dist)) for r in range(n)]
        outs, _ = ref.reduce_scatter(ins, DT[dtype][1])
        save(f"reduce_scatter_n{n}_{dtype}_{rows}x{cols}", ins, outs,
             {"op": "reduce_scatter", "n": n, "dtype": dtype, "rows": rows, "cols": cols})
        cases += 1
    # Shard(d) -> Replicate, even and uneven (the reference test's (4,8) and (5,9) shapes included)
    for n, dtype, full, dim in [(2, "float32", (4, 8), 0), (2, "float32", (5, 9), 0), (2, "float32", (5, 9), 1),
                                (4, "bfloat16", (2, 16, 12), 2), (3, "float16", (7, 5, 3), 0),
                                (8, "float32", (3, 19, 4), 1), (8, "bfloat16", (64, 32), 0)]:
        lens = shard_sizes(full[dim], n)
        ins = []
        for r in range(n):
            shp = list(full)
            shp[dim] = lens[r]
            ins.append(raw(gen(shp, dtype, 300 + r, "rand")))
        outs, _ = ref.all_gather(ins, DT[dtype][1], dim)
        save(f"all_gather_n{n}_{dtype}_{'x'.join(map(str, full))}_d{dim}", ins, outs,
             {"op": "all_gather", "n": n, "dtype": dtype, "dim": dim})
        cases += 1
    # Shard(i) -> Shard(j) (the reference test's S1<->S0 on (4,8)/(5,9), a Ulysses-shaped case, odd shapes)
    for n, dtype, full, sd, dd in [(2, "float32", (4, 8), 0, 1), (2, "float32", (5, 9), 1, 0),
                                   (2, "float32", (5, 9), 0, 1), (4, "bfloat16", (1, 16, 8, 4), 1, 2),
                                   (4, "bfloat16", (1, 8, 16, 4), 2, 1), (8, "float16", (16, 11, 13, 3), 2, 0),
                                   (3, "float32", (6, 7, 5), 0, 2), (8, "bfloat16", (1, 32, 16, 8), 1, 2)]:
        lens = shard_sizes(full[sd], n)
        ins = []
        for r in range(n):
            shp = list(full)
            shp[sd] = lens[r]
            ins.append(raw(gen(shp, dtype, 400 + r, "randn")))
        outs, _ = ref.all_to_all(ins, DT[dtype][1], sd, dd)
        save(f"all_to_all_n{n}_{dtype}_{'x'.join(map(str, full))}_s{sd}_d{dd}", ins, outs,
             {"op": "all_to_all", "n": n, "dtype": dtype, "src_dim": sd, "dst_dim": dd})
        cases += 1
    print(f"wrote {cases} golden cases to {HERE}")


if __name__ == "__main__":
    main()
