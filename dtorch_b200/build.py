"""In-tree build of the native parts of dtorch_b200 (run: ``python -m dtorch_b200.build``).

* ``_lib/libdtorch_b200.so`` -- the C ABI (include/dtorch_b200.h) and its sm_100a kernels, compiled by nvcc
  with ``-gencode arch=compute_100a,code=sm_100a``; the CUDA runtime is linked statically so the library does
  not depend on which libcudart the host process loaded first.
* ``_host.so`` -- the C++ host layer (ThreadGroup, c10d backend, kernel-stream threads, redistribute
  executor, placement algebra) as a Python extension, linked against libtorch and ``_lib/libdtorch_b200.so``.
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


HOST_SRCS = ["placement.cpp", "sym_pool.cpp", "thread_group.cpp", "redistribute.cpp", "bindings.cpp"]


def build_host(force: bool = False, verbose: bool = False) -> str:
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    hostdir = os.path.join(CSRC, "host")
    out = os.path.join(HERE, "_host" + sysconfig.get_config_var("EXT_SUFFIX"))
    srcs = [os.path.join(hostdir, f) for f in sorted(os.listdir(hostdir))]
    srcs += [os.path.join(ROOT, "include", "dtorch_b200.h"), os.path.join(LIBDIR, "libdtorch_b200.so")]
    if not (force or _newer(out, srcs)):
        return out
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{cuda_home}/include",
                                                               f"-I{sysconfig.get_paths()['include']}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = ["-O2", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
             "-DTORCH_EXTENSION_NAME=_host", "-DPYBIND11_COMPILER_TYPE=\"_gcc\"", "-DPYBIND11_STDLIB=\"_libstdcpp\"",
             "-DPYBIND11_BUILD_ABI=\"_cxxabi1018\"", "-fvisibility=hidden", "-Wall", "-Wno-unused-function",
             "-Wno-interference-size"]
    objs = []
    procs = []
    for f in HOST_SRCS:
        obj = os.path.join(objdir, f.replace(".cpp", ".o"))
        objs.append(obj)
        cmd = ["g++", *flags, *incs, "-c", os.path.join(hostdir, f), "-o", obj]
        if verbose:
            print(" ".join(cmd[:3]), "...", f, flush=True)
        procs.append(subprocess.Popen(cmd))
    if any(p.wait() != 0 for p in procs):
        raise RuntimeError("host extension compile failed")
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    link = ["g++", "-shared", "-o", out + ".tmp", *objs, f"-L{torch_lib}", f"-Wl,-rpath,{torch_lib}",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            f"-L{LIBDIR}", "-ldtorch_b200", "-Wl,-rpath,$ORIGIN/_lib"]
    subprocess.run(link, check=True)
    os.replace(out + ".tmp", out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_capi(force=force, verbose=verbose)
    build_host(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
