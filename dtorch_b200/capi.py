"""ctypes binding of the C ABI in include/dtorch_b200.h (libdtorch_b200.so, built in-tree).

This is the boundary the parity tests and the bench call through: plain pointers, sizes and a cudaStream_t.
There is no fallback: if the library is missing, importing raises, so a CUDA path can never silently turn
into something else.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libdtorch_b200.so")

DT_OK = 0
DT_ERR_INVALID = 1
DT_ERR_CUDA = 2
DT_ERR_TIMEOUT = 3
DT_ERR_PEER = 4
DT_ERR_UNSUPPORTED = 5
DT_ERR_STATE = 6

DT_FLOAT32, DT_BFLOAT16, DT_FLOAT16 = 0, 1, 2
DT_SUM = 0
DT_ACCUM_FP32 = 0x0
DT_ACCUM_STORAGE = 0x1
DT_RANK_ORDER = 0x2
DT_ALGO_ONESHOT = 0x10
DT_ALGO_TWOSHOT = 0x20
DT_ALGO_NVLS = 0x40
DT_ALGO_NCCL = 0x80

MAX_RANKS = 8

# (name, restype, argtypes) of every exported entry point; the CPU test suite checks this list against the
# declarations in include/dtorch_b200.h.
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_I64 = ctypes.c_int64
SIGNATURES = [
    ("dt_status_string", ctypes.c_char_p, [_I]),
    ("dt_last_error_message", ctypes.c_char_p, []),
    ("dt_version", _I, []),
    ("dt_comm_create", _I, [_I, _P, _SZ, _P]),
    ("dt_comm_create_rank", _I, [_I, _I, _I, _SZ, _P]),
    ("dt_comm_handle_bytes", _SZ, []),
    ("dt_comm_export", _I, [_P, _P]),
    ("dt_comm_import", _I, [_P, _P]),
    ("dt_comm_destroy", _I, [_P]),
    ("dt_comm_size", _I, [_P]),
    ("dt_comm_same_device", _I, [_P]),
    ("dt_comm_heap", _I, [_P, _I, _P, _P]),
    ("dt_comm_set_timeout_ms", _I, [_P, _I64]),
    ("dt_comm_error", _I, [_P, _I]),
    ("dt_comm_clear_error", _I, [_P, _I]),
    ("dt_all_reduce", _I, [_P, _I, _P, _P, _SZ, _I, _I, _I, _P]),
    ("dt_reduce_scatter", _I, [_P, _I, _P, _P, _SZ, _I, _I, _I, _P]),
    ("dt_all_gather", _I, [_P, _I, _P, _P, _SZ, _P, _SZ, _P]),
    ("dt_all_to_all", _I, [_P, _I, _P, _P, _I, _P, _I, _I, _P, _SZ, _P]),
    ("dt_barrier", _I, [_P, _I, _P]),
    ("dt_local_all_reduce", _I, [_I, _P, _P, _SZ, _I, _I, _P]),
    ("dt_local_all_reduce_host", _I, [_I, _P, _P, _P, _P, _SZ, _I, _I, _SZ, _P]),
    ("dt_local_reduce_scatter", _I, [_I, _P, _P, _SZ, _I, _I, _P]),
    ("dt_local_all_gather", _I, [_I, _P, _P, _SZ, _P, _SZ, _P]),
    ("dt_local_all_to_all", _I, [_I, _P, _P, _I, _P, _I, _I, _P, _SZ, _P]),
    ("dt_kernel_launch_count", ctypes.c_uint64, []),
    ("dt_all_to_all_multi", _I, [_P, _I, _I, _P, _P, _I, _P, _I, _I, _P, _SZ, _P]),
    ("dt_comm_nvls_supported", _I, [_P, _P]),
    ("dt_comm_nvls_alloc", _I, [_P, _SZ]),
    ("dt_comm_nvls_create", _I, [_P, _SZ, _P]),
    ("dt_comm_nvls_attach", _I, [_P, _I, _SZ]),
    ("dt_comm_nvls_bind", _I, [_P]),
    ("dt_comm_nvls_buffer", _I, [_P, _I, _P, _P]),
    ("dt_local_all_reduce_host_noalloc", _I, [_I, _P, _P, _SZ, _I, _I, _P]),
    ("dt_all_to_all_list", _I, [_P, _I, _P, _P, _P, _P, _P]),
    ("dt_all_gather_list", _I, [_P, _I, _P, _SZ, _P, _P, _P]),
    ("dt_all_gather_sub_split", _I, [_P, _I, _P, _P, _SZ, _P, _P, _SZ, _P]),
    ("dt_peer_copy", _I, [_P, _I, _P, _I, _SZ, _P]),
]


class DtError(RuntimeError):
    """A dt_* entry point returned a non-zero status."""

    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)} ({detail})")
        self.status = status


STATUS_NAMES = {
    DT_OK: "ok",
    DT_ERR_INVALID: "DT_ERR_INVALID",
    DT_ERR_CUDA: "DT_ERR_CUDA",
    DT_ERR_TIMEOUT: "DT_ERR_TIMEOUT",
    DT_ERR_PEER: "DT_ERR_PEER",
    DT_ERR_UNSUPPORTED: "DT_ERR_UNSUPPORTED",
    DT_ERR_STATE: "DT_ERR_STATE",
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libdtorch_b200.so once and declare every signature. Raises if the library was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m dtorch_b200.build` "
                              "(there is no fallback path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, where: str) -> None:
    if status != DT_OK:
        detail = lib().dt_last_error_message().decode(errors="replace")
        raise DtError(status, where, detail)


def ptr_array(ptrs: Sequence[int]):
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


def size_array(vals: Sequence[int]):
    return (ctypes.c_size_t * len(vals))(*[int(v) for v in vals])


def i64_array(vals: Sequence[int]):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def launch_count() -> int:
    return int(lib().dt_kernel_launch_count())


def dtype_code(torch_dtype) -> int:
    import torch

    codes = {torch.float32: DT_FLOAT32, torch.bfloat16: DT_BFLOAT16, torch.float16: DT_FLOAT16}
    if torch_dtype not in codes:
        raise TypeError(f"unsupported dtype for a reduction: {torch_dtype}")
    return codes[torch_dtype]


class Comm:
    """A dt_comm handle. Single-process (``Comm(devices)``) or one rank of a multi-process group
    (``Comm.for_rank(n, rank, device)`` then ``export_handle`` / ``import_handles``)."""

    def __init__(self, devices: Optional[Sequence[int]] = None, heap_bytes: int = 0, _handle=None):
        self._h = ctypes.c_void_p()
        if _handle is not None:
            self._h = _handle
        else:
            devs = (ctypes.c_int * len(devices))(*devices)
            check(lib().dt_comm_create(len(devices), devs, heap_bytes, ctypes.byref(self._h)), "dt_comm_create")
        self.n = lib().dt_comm_size(self._h)
        self.same_device = bool(lib().dt_comm_same_device(self._h))

    @classmethod
    def for_rank(cls, n: int, rank: int, device: int, heap_bytes: int) -> "Comm":
        h = ctypes.c_void_p()
        check(lib().dt_comm_create_rank(n, rank, device, heap_bytes, ctypes.byref(h)), "dt_comm_create_rank")
        return cls(_handle=h)

    @property
    def handle(self):
        return self._h

    def export_handle(self) -> bytes:
        nb = lib().dt_comm_handle_bytes()
        buf = ctypes.create_string_buffer(nb)
        check(lib().dt_comm_export(self._h, buf), "dt_comm_export")
        return buf.raw

    def import_handles(self, handles: Sequence[bytes]) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(lib().dt_comm_import(self._h, buf), "dt_comm_import")

    def heap(self, rank: int):
        base = ctypes.c_void_p()
        size = ctypes.c_size_t()
        check(lib().dt_comm_heap(self._h, rank, ctypes.byref(base), ctypes.byref(size)), "dt_comm_heap")
        return base.value or 0, size.value

    # ---- NVLS buffer ----
    def nvls_supported(self) -> bool:
        v = ctypes.c_int()
        check(lib().dt_comm_nvls_supported(self._h, ctypes.byref(v)), "dt_comm_nvls_supported")
        return bool(v.value)

    def nvls_alloc(self, nbytes: int) -> None:
        check(lib().dt_comm_nvls_alloc(self._h, nbytes), "dt_comm_nvls_alloc")

    def nvls_create(self, nbytes: int) -> int:
        fd = ctypes.c_int(-1)
        check(lib().dt_comm_nvls_create(self._h, nbytes, ctypes.byref(fd)), "dt_comm_nvls_create")
        return fd.value

    def nvls_attach(self, fd: int, nbytes: int) -> None:
        check(lib().dt_comm_nvls_attach(self._h, fd, nbytes), "dt_comm_nvls_attach")

    def nvls_bind(self) -> None:
        check(lib().dt_comm_nvls_bind(self._h), "dt_comm_nvls_bind")

    def nvls_buffer(self, rank: int):
        base = ctypes.c_void_p()
        size = ctypes.c_size_t()
        check(lib().dt_comm_nvls_buffer(self._h, rank, ctypes.byref(base), ctypes.byref(size)), "dt_comm_nvls_buffer")
        return base.value or 0, size.value

    def set_timeout_ms(self, ms: int) -> None:
        check(lib().dt_comm_set_timeout_ms(self._h, ms), "dt_comm_set_timeout_ms")

    def error(self, rank: int) -> int:
        return lib().dt_comm_error(self._h, rank)

    def clear_error(self, rank: int) -> None:
        check(lib().dt_comm_clear_error(self._h, rank), "dt_comm_clear_error")

    def destroy(self) -> None:
        if self._h:
            lib().dt_comm_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    # ---- collectives (raw pointers) ----
    def all_reduce(self, rank, inp, out, count, dtype, flags=0, stream=0):
        check(lib().dt_all_reduce(self._h, rank, inp, out, count, dtype, DT_SUM, flags, stream), "dt_all_reduce")

    def reduce_scatter(self, rank, inp, out, out_count, dtype, flags=0, stream=0):
        check(lib().dt_reduce_scatter(self._h, rank, inp, out, out_count, dtype, DT_SUM, flags, stream),
              "dt_reduce_scatter")

    def all_gather(self, rank, inp, out, outer, lens, inner_bytes, stream=0):
        check(lib().dt_all_gather(self._h, rank, inp, out, outer, i64_array(lens), inner_bytes, stream),
              "dt_all_gather")

    def all_gather_sub_split(self, rank, inp, out, outer, lens, fronts, inner_bytes, stream=0):
        check(lib().dt_all_gather_sub_split(self._h, rank, inp, out, outer, i64_array(lens), i64_array(fronts),
                                            inner_bytes, stream), "dt_all_gather_sub_split")

    def all_to_all(self, rank, inp, out, in_shape, src_dim, dst_dim, src_lens, elem_bytes, stream=0):
        check(lib().dt_all_to_all(self._h, rank, inp, out, len(in_shape), i64_array(in_shape), src_dim, dst_dim,
                                  i64_array(src_lens), elem_bytes, stream), "dt_all_to_all")

    def all_to_all_multi(self, rank, ins, outs, in_shape, src_dim, dst_dim, src_lens, elem_bytes, stream=0):
        check(lib().dt_all_to_all_multi(self._h, rank, len(ins), ptr_array(ins), ptr_array(outs), len(in_shape),
                                        i64_array(in_shape), src_dim, dst_dim, i64_array(src_lens), elem_bytes, stream),
              "dt_all_to_all_multi")

    def all_to_all_list(self, rank, ins, in_bytes, outs, out_bytes, stream=0):
        check(lib().dt_all_to_all_list(self._h, rank, ptr_array(ins), size_array(in_bytes), ptr_array(outs),
                                       size_array(out_bytes), stream), "dt_all_to_all_list")

    def all_gather_list(self, rank, inp, in_bytes, outs, out_bytes, stream=0):
        check(lib().dt_all_gather_list(self._h, rank, inp, in_bytes, ptr_array(outs), size_array(out_bytes), stream),
              "dt_all_gather_list")

    def barrier(self, rank, stream=0):
        check(lib().dt_barrier(self._h, rank, stream), "dt_barrier")


# ---- same-device kernels ----
def local_all_reduce(ins, out, count, dtype, flags=0, stream=0):
    check(lib().dt_local_all_reduce(len(ins), ptr_array(ins), out, count, dtype, flags, stream), "dt_local_all_reduce")


def local_all_reduce_host(host_ins, dev_ins, dev_out, host_out, count, dtype, flags=0, chunk_bytes=0, stream=0):
    """Same-device all-reduce of pinned host partials, staged through device buffers chunk by chunk with the
    copies in both directions overlapping the reduction; host_out is complete when `stream` reaches the call's end."""
    check(lib().dt_local_all_reduce_host(len(host_ins), ptr_array(host_ins), ptr_array(dev_ins), dev_out, host_out,
                                         count, dtype, flags, chunk_bytes, stream), "dt_local_all_reduce_host")


def peer_copy(dst, dst_device, src, src_device, nbytes, stream=0):
    """Kernel copy from src_device's memory into dst_device's over NVLink, on src_device's `stream`."""
    check(lib().dt_peer_copy(dst, dst_device, src, src_device, nbytes, stream), "dt_peer_copy")


NOALLOC_SCRATCH_BYTES = 32 << 20  # DT_NOALLOC_SCRATCH_BYTES


def local_all_reduce_host_noalloc(host_ins, host_out, count, dtype, flags=0, stream=0):
    """dt_local_all_reduce_host without staging buffers: the partials and the sum pass through the library's
    fixed device scratch (NOALLOC_SCRATCH_BYTES per GPU), for callers that cannot allocate device memory.
    (n + 1) slots of count * element size bytes, each rounded up to 256, must fit; calls that overlap on the
    GPU race on the shared scratch."""
    check(lib().dt_local_all_reduce_host_noalloc(len(host_ins), ptr_array(host_ins), host_out, count, dtype, flags,
                                                 stream), "dt_local_all_reduce_host_noalloc")


def local_reduce_scatter(ins, outs, out_count, dtype, flags=0, stream=0):
    check(lib().dt_local_reduce_scatter(len(ins), ptr_array(ins), ptr_array(outs), out_count, dtype, flags, stream),
          "dt_local_reduce_scatter")


def local_all_gather(ins, out, outer, lens, inner_bytes, stream=0):
    check(lib().dt_local_all_gather(len(ins), ptr_array(ins), out, outer, i64_array(lens), inner_bytes, stream),
          "dt_local_all_gather")


def local_all_to_all(ins, outs, in_shape, src_dim, dst_dim, src_lens, elem_bytes, stream=0):
    check(lib().dt_local_all_to_all(len(ins), ptr_array(ins), ptr_array(outs), len(in_shape), i64_array(in_shape),
                                    src_dim, dst_dim, i64_array(src_lens), elem_bytes, stream), "dt_local_all_to_all")
