"""Shared helpers of the test suite: golden fixtures, raw <-> torch conversion, tolerances."""

import glob
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT_CODE = {"float32": 0, "bfloat16": 1, "float16": 2}

# Tolerance for reductions computed with fp32 accumulation against the reference's in-dtype fold
# (north star: rel 1e-6 for fp32, rel 2e-2 for bf16/fp16; measured as allclose(rtol, atol = rtol * rms(ref))).
RTOL = {"float32": 1e-6, "bfloat16": 2e-2, "float16": 2e-2}


def golden_cases(op=None):
    out = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        z = np.load(path)
        meta = json.loads(bytes(z["meta"]).decode())
        if op is not None and meta["op"] != op:
            continue
        n = meta["n"]
        ins = [z[f"in_{r}"] for r in range(n)]
        outs = [z[f"out_{r}"] for r in range(n)]
        out.append((os.path.basename(path)[:-4], meta, ins, outs))
    return out


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return a.astype(np.float32)
    if dtype == "bfloat16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


def assert_close(got: np.ndarray, ref: np.ndarray, dtype: str):
    g = to_f32(got, dtype).astype(np.float64)
    r = to_f32(ref, dtype).astype(np.float64)
    rtol = RTOL[dtype]
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    atol = rtol * rms
    bad = np.abs(g - r) > atol + rtol * np.abs(r)
    assert not bad.any(), f"{int(bad.sum())} / {bad.size} elements outside rtol={rtol} atol={atol:g}"


def abs_sum_f64(ins, dtype: str) -> np.ndarray:
    """Per-element sum of |x_r| over the ranks' partials: the scale of the rounding error of any floating-point
    summation of them (recursive summation of n terms errs by at most (n-1)·u·sum|x_r|, Higham, Accuracy and
    Stability of Numerical Algorithms, section 4.2)."""
    acc = np.zeros(ins[0].size, dtype=np.float64)
    for a in ins:
        acc += np.abs(to_f32(a.reshape(-1), dtype))
    return acc


def exact_sum_f64(ins, dtype: str) -> np.ndarray:
    acc = np.zeros(ins[0].size, dtype=np.float64)
    for a in ins:
        acc += to_f32(a.reshape(-1), dtype)
    return acc


def assert_close_sum(got: np.ndarray, ref: np.ndarray, dtype: str, abs_sum: np.ndarray):
    """|got - ref| <= rtol * sum_r |x_r| element by element: two summations of the same partials (here fp32
    accumulation vs the reference's per-add rounding to bf16/fp16) agree to the error scale of summation itself.
    At 64 M elements the rms-scaled form of assert_close flags the rare element where the reference's seven bf16
    roundings drift on large partial sums that cancel; this scale follows the partial sums."""
    g = to_f32(got.reshape(-1), dtype).astype(np.float64)
    r = to_f32(ref.reshape(-1), dtype).astype(np.float64)
    rtol = RTOL[dtype]
    bad = np.abs(g - r) > rtol * abs_sum
    assert not bad.any(), f"{int(bad.sum())} / {bad.size} elements outside rtol={rtol} of sum|x|"


def torch_from_raw(a: np.ndarray, dtype: str, device="cpu"):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype == "bfloat16":
        t = t.view(torch.int16).view(torch.bfloat16)
    elif dtype == "float16":
        t = t.view(torch.int16).view(torch.float16)
    return t.to(device)


def raw_from_torch(t) -> np.ndarray:
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()
