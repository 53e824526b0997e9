"""CPU: the C-ABI library loads without a GPU and exports every entry point include/dtorch_b200.h declares,
with the signature table of the Python binding covering exactly those entry points."""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

from dtorch_b200 import capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "dtorch_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(dt_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "dt_all_reduce" in names and "dt_all_to_all" in names and "dt_comm_create" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(capi.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_matches_header():
    assert sorted(n for n, _, _ in capi.SIGNATURES) == declared_functions()


def test_host_only_calls():
    L = capi.lib()
    assert L.dt_version() >> 16 == 1
    assert L.dt_status_string(capi.DT_ERR_TIMEOUT) == b"timeout waiting for a peer"
    assert L.dt_comm_handle_bytes() >= 64
    # invalid arguments are rejected before any CUDA call
    assert L.dt_comm_create(0, None, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_all_reduce(None, 0, None, None, 0, 0, 0, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_local_all_reduce(0, None, None, 0, 0, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_local_all_reduce(2, None, None, 16, 9, 0, None) == capi.DT_ERR_INVALID


def test_all_to_all_rejects_dst_extent_below_group():
    # The reference asserts shapeSize >= numShard in GetShardSizeForAllRank (distributed_spec.cc:203, active in
    # its default DTORCH_DEBUG build) and CheckValid rejects such placements; the C ABI refuses them too,
    # before touching the device.
    L = capi.lib()
    dummy = capi.ptr_array([16] * 8)
    shape = capi.i64_array([2, 11, 2, 3])
    lens = capi.i64_array([2, 2, 2, 2, 2, 1, 1, 1])
    assert L.dt_local_all_to_all(8, dummy, dummy, 4, shape, 2, 0, lens, 2, None) == capi.DT_ERR_INVALID
    assert b"dst dim" in L.dt_last_error_message()


def test_host_buffer_all_reduce_rejects_bad_arguments():
    L = capi.lib()
    ptrs = capi.ptr_array([16] * 2)
    assert L.dt_local_all_reduce_host(0, ptrs, ptrs, 16, 16, 8, 0, 0, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_local_all_reduce_host(2, ptrs, ptrs, 16, 16, 8, 7, 0, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_local_all_reduce_host(2, ptrs, ptrs, None, 16, 8, 0, 0, 0, None) == capi.DT_ERR_INVALID
    assert L.dt_local_all_reduce_host(2, ptrs, ptrs, 16, 16, 0, 0, 0, 0, None) == capi.DT_OK  # nothing to do


def test_header_is_plain_c_and_links(tmp_path):
    """A C program (no C++, no torch) includes the header, links the library and makes host-only calls: the
    boundary is a plain C ABI."""
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "abi.c"
    src.write_text(
        '#include <stdio.h>\n#include "dtorch_b200.h"\n'
        "int main(void) {\n"
        "  dt_comm* c = 0;\n"
        "  if (dt_comm_create(0, 0, 0, &c) != DT_ERR_INVALID) return 1;\n"
        '  printf("%d %s\\n", dt_version() >> 16, dt_status_string(DT_ERR_TIMEOUT));\n'
        "  return 0;\n}\n")
    exe = tmp_path / "abi"
    libdir = os.path.dirname(capi.LIB_PATH)
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", f"-I{os.path.dirname(HEADER)}", str(src), "-o", str(exe),
                    f"-L{libdir}", "-ldtorch_b200", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert out.strip() == "1 timeout waiting for a peer"


def test_flag_constants_match_header():
    text = open(HEADER).read()
    defines = dict(re.findall(r"^#define\s+(DT_[A-Z0-9_]+)\s+(0x[0-9a-fA-F]+|\d+)\s*$", text, flags=re.M))
    flags = {k: int(v, 0) for k, v in defines.items() if k.startswith(("DT_ALGO_", "DT_ACCUM_", "DT_RANK_"))}
    assert {"DT_ALGO_NCCL", "DT_RANK_ORDER", "DT_ALGO_NVLS", "DT_ACCUM_STORAGE"} <= set(flags)
    for name, value in flags.items():
        if name == "DT_ALGO_AUTO":
            continue
        assert getattr(capi, name) == value, name
    # the reduction flags are distinct bits
    bits = [v for k, v in flags.items() if v]
    assert len(bits) == len(set(bits)) and all(v & (v - 1) == 0 for v in bits)
