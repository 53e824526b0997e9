"""GPU-side helpers of the test suite (imported only by -m gpu tests)."""

import threading

import numpy as np
import torch

from dtorch_b200 import capi
from tests.helpers import raw_from_torch, torch_from_raw


class _CAI:
    """Expose a raw device pointer through __cuda_array_interface__ so torch can view it."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


def view_device_memory(ptr: int, numel: int, dtype, device: int) -> torch.Tensor:
    ts = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.float16: "<i2", torch.uint8: "|u1"}[dtype]
    with torch.cuda.device(device):
        t = torch.as_tensor(_CAI(ptr, (numel,), ts), device=f"cuda:{device}")
    if dtype in (torch.bfloat16, torch.float16):
        t = t.view(dtype)
    return t


def to_dev(a: np.ndarray, dtype: str, device: int) -> torch.Tensor:
    return torch_from_raw(a, dtype, f"cuda:{device}")


def run_ranks(n, fn):
    """Run fn(rank) on n threads (one per rank, as the reference's rank threads); re-raise the first error."""
    errs = [None] * n

    def body(r):
        try:
            fn(r)
        except BaseException as e:  # noqa: BLE001
            errs[r] = e

    th = [threading.Thread(target=body, args=(r,)) for r in range(n)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    for t in th:
        assert not t.is_alive(), "rank thread did not finish"
    for e in errs:
        if e is not None:
            raise e


def np_raw(t) -> np.ndarray:
    return raw_from_torch(t)


def stream_ptr(s: torch.cuda.Stream) -> int:
    return s.cuda_stream


def launches() -> int:
    return capi.launch_count()
