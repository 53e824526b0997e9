"""In-tree build of the native parts of dtorch_b200 (run: ``python -m dtorch_b200.build``).

* ``_lib/libdtorch_b200.so`` -- the C ABI (include/dtorch_b200.h) and its sm_100a kernels, compiled by nvcc
  with ``-gencode arch=compute_100a,code=sm_100a``; the CUDA runtime is linked statically so the library does
  not depend on which libcudart the host process loaded first.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def _newer(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_capi(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    out = os.path.join(LIBDIR, "libdtorch_b200.so")
    srcs = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".h"))]
    srcs.append(os.path.join(ROOT, "include", "dtorch_b200.h"))
    if force or _newer(out, srcs):
        cmd = [nvcc(), *NVCC_FLAGS, *ARCH, "-shared", "-cudart", "static", "-o", out + ".tmp",
               os.path.join(CSRC, "dt_comm.cu")]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_capi(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
