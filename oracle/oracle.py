"""TEST INFRASTRUCTURE ONLY -- the CPU oracles of the redistribute collectives.

Two checkers, both on the host:

* ``Restatement`` wraps ``liboracle.so`` (dt_oracle.c): a plain-C restatement of what the reference's
  same-device thread-group backend computes (thread_group_same_device_backend.cc:111-302,
  thread_group.cc:127-241, distributed_spec.cc:202-213).
* ``Reference`` wraps ``_ref/libdtref.so``: the reference's own ThreadGroup / ThreadGroupSameDeviceBackend /
  MemoryTensorStore sources compiled out of tree (oracle/Makefile, target ``ref``), driven by n rank threads
  on a CPU DeviceMesh exactly as the reference drives them. It exists where the reference sources were
  present at build time.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm use this module; the
product path never imports it.

Arrays are numpy arrays holding the raw storage: float32 for fp32, uint16 bit patterns for bf16 / fp16
(``dtype`` codes 0 / 1 / 2 as in include/dtorch_b200.h).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libdtref.so")

DTYPES = {"float32": 0, "bfloat16": 1, "float16": 2}
NP_STORAGE = {0: np.float32, 1: np.uint16, 2: np.uint16}
ELEM_BYTES = {0: 4, 1: 2, 2: 2}


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and the reference library when ``ref`` and the sources are present)."""
    subprocess.run(["make", "-s", "liboracle.so"], cwd=HERE, check=True)
    if ref:
        subprocess.run(["make", "-s", "-j8", "ref"], cwd=HERE, check=True)


def _ptrs(arrays: Sequence[Optional[np.ndarray]]):
    arr = (ctypes.c_void_p * len(arrays))()
    for i, a in enumerate(arrays):
        arr[i] = None if a is None else a.ctypes.data
    return arr


def _i64(vals: Sequence[int]):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def _contig(a: np.ndarray, dtype: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype != NP_STORAGE[dtype]:
        raise TypeError(f"storage of dtype code {dtype} must be {NP_STORAGE[dtype]}, got {a.dtype}")
    return a


def shard_sizes(length: int, n: int) -> List[int]:
    """Placement::GetShardSizeForAllRank (distributed_spec.cc:202-213): first length % n ranks get one more."""
    return [length // n + (1 if i < length % n else 0) for i in range(n)]


class Restatement:
    """ctypes binding of dt_oracle.c."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.oracle_fold_sum.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
        L.oracle_reduce_scatter.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
        L.oracle_all_gather.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        L.oracle_all_to_all.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_bf16_to_f32.restype = ctypes.c_float
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f16_to_f32.restype = ctypes.c_float

    def fold_sum(self, ins: Sequence[np.ndarray], dtype: int, storage_round: bool = True) -> np.ndarray:
        ins = [_contig(a, dtype) for a in ins]
        out = np.empty_like(ins[0])
        self.lib.oracle_fold_sum(len(ins), _ptrs(ins), out.ctypes.data, ins[0].size, dtype, int(storage_round))
        return out

    def reduce_scatter(self, ins: Sequence[np.ndarray], dtype: int, storage_round: bool = True) -> List[np.ndarray]:
        ins = [_contig(a, dtype) for a in ins]
        n = len(ins)
        if ins[0].shape[0] % n:
            raise ValueError("reduce-scatter needs dim 0 divisible by the group size (thread_group.cc:195)")
        out_shape = (ins[0].shape[0] // n,) + ins[0].shape[1:]
        outs = [np.empty(out_shape, dtype=ins[0].dtype) for _ in range(n)]
        self.lib.oracle_reduce_scatter(n, _ptrs(ins), _ptrs(outs), outs[0].size, dtype, int(storage_round))
        return outs

    def all_gather(self, ins: Sequence[np.ndarray], dim: int) -> np.ndarray:
        ins = [np.ascontiguousarray(a) for a in ins]
        shape = list(ins[0].shape)
        outer = int(np.prod(shape[:dim], dtype=np.int64))
        inner = int(np.prod(shape[dim + 1:], dtype=np.int64)) * ins[0].itemsize
        lens = [a.shape[dim] for a in ins]
        shape[dim] = sum(lens)
        out = np.empty(shape, dtype=ins[0].dtype)
        self.lib.oracle_all_gather(len(ins), _ptrs(ins), out.ctypes.data, outer, _i64(lens), inner)
        return out

    def all_to_all(self, ins: Sequence[np.ndarray], src_dim: int, dst_dim: int,
                   only: Optional[int] = None) -> List[Optional[np.ndarray]]:
        """Every rank's output, or with ``only=k`` rank k's alone (the other entries are None)."""
        ins = [np.ascontiguousarray(a) for a in ins]
        n = len(ins)
        src_lens = [a.shape[src_dim] for a in ins]
        D = ins[0].shape[dst_dim]
        split = shard_sizes(D, n)
        outs = []
        for k in range(n):
            if only is not None and k != only:
                outs.append(None)
                continue
            shp = list(ins[0].shape)
            shp[src_dim] = sum(src_lens)
            shp[dst_dim] = split[k]
            outs.append(np.empty(shp, dtype=ins[0].dtype))
        self.lib.oracle_all_to_all(n, _ptrs(ins), _ptrs(outs), ins[0].ndim, _i64(ins[0].shape), src_dim, dst_dim,
                                   _i64(src_lens), ins[0].itemsize)
        return outs


class Reference:
    """ctypes binding of the reference's own ThreadGroup on a CPU DeviceMesh (oracle/_ref/libdtref.so)."""

    def __init__(self, path: str = REF_LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (make -C oracle ref, needs the reference sources)")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.dtref_last_error.restype = ctypes.c_char_p
        L.dtref_all_reduce.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.dtref_reduce_scatter.argtypes = L.dtref_all_reduce.argtypes
        L.dtref_all_gather.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.dtref_all_to_all.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p]

    @staticmethod
    def available(path: str = REF_LIB_PATH) -> bool:
        return os.path.exists(path)

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(f"reference harness failed ({rc}): {self.lib.dtref_last_error().decode()}")

    def all_reduce(self, ins, dtype: int, iters: int = 1, threads: int = 0):
        ins = [_contig(a, dtype).reshape(-1) for a in ins]
        outs = [np.empty_like(ins[0]) for _ in ins]
        secs = np.zeros(iters, dtype=np.float64)
        self._check(self.lib.dtref_all_reduce(len(ins), dtype, _ptrs(ins), _ptrs(outs), ins[0].size, iters, threads,
                                              secs.ctypes.data))
        return outs, secs

    def reduce_scatter(self, ins, dtype: int, iters: int = 1, threads: int = 0):
        n = len(ins)
        ins = [_contig(a, dtype).reshape(-1) for a in ins]
        out_count = ins[0].size // n
        outs = [np.empty(out_count, dtype=ins[0].dtype) for _ in ins]
        secs = np.zeros(iters, dtype=np.float64)
        self._check(self.lib.dtref_reduce_scatter(n, dtype, _ptrs(ins), _ptrs(outs), out_count, iters, threads,
                                                  secs.ctypes.data))
        return outs, secs

    def all_gather(self, ins, dtype: int, dim: int, iters: int = 1, threads: int = 0):
        ins = [_contig(a, dtype) for a in ins]
        n, ndim = len(ins), ins[0].ndim
        shapes = [s for a in ins for s in a.shape]
        out_shape = list(ins[0].shape)
        out_shape[dim] = sum(a.shape[dim] for a in ins)
        outs = [np.empty(out_shape, dtype=ins[0].dtype) for _ in ins]
        secs = np.zeros(iters, dtype=np.float64)
        self._check(self.lib.dtref_all_gather(n, dtype, _ptrs(ins), _ptrs(outs), ndim, _i64(shapes), dim, iters,
                                              threads, secs.ctypes.data))
        return outs, secs

    def all_to_all(self, ins, dtype: int, src_dim: int, dst_dim: int, iters: int = 1, threads: int = 0):
        ins = [_contig(a, dtype) for a in ins]
        n, ndim = len(ins), ins[0].ndim
        if ins[0].shape[dst_dim] < n:
            # the reference asserts shapeSize >= numShard (distributed_spec.cc:203) and its harness would exit
            raise ValueError("all-to-all: destination extent smaller than the group")
        shapes = [s for a in ins for s in a.shape]
        split = shard_sizes(ins[0].shape[dst_dim], n)
        outs = []
        for k in range(n):
            shp = list(ins[0].shape)
            shp[src_dim] = sum(a.shape[src_dim] for a in ins)
            shp[dst_dim] = split[k]
            outs.append(np.empty(shp, dtype=ins[0].dtype))
        secs = np.zeros(iters, dtype=np.float64)
        self._check(self.lib.dtref_all_to_all(n, dtype, _ptrs(ins), _ptrs(outs), ndim, _i64(shapes), src_dim, dst_dim,
                                              iters, threads, secs.ctypes.data))
        return outs, secs
