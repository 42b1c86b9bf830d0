"""The native library builds for sm_100a and loads on a host without a GPU."""

import ctypes
import os
from pathlib import Path

import pytest
import torch

from numa_allreduce_b200.ops import _ext


def test_torch_ops_load_and_layout():
    ops = _ext.load()
    assert _ext.loaded_path().endswith("_C.so")
    assert ops.meta_size() > 0
    ws_bytes, mc_bytes, one, two, hier, fused, pipe = ops.layout(8, [1 << 20, 64 << 10, 64, 32, 512 << 10])
    assert 0 < one < two < hier < pipe < fused < ws_bytes
    assert mc_bytes > 0
    assert all(v % 4096 == 0 for v in (one, two, hier, fused, pipe))
    with pytest.raises((RuntimeError, ValueError)):
        ops.layout(9, [])
    with pytest.raises((RuntimeError, ValueError)):
        ops.layout(8, [1 << 20, 100])
    with pytest.raises((RuntimeError, ValueError)):
        ops.layout(8, [1 << 20, 0, 128, 32, 512 << 10, 1, 128, 1000])  # pipe tile too small


def test_c_abi_exports():
    _ext.load()
    lib = ctypes.CDLL(str(_ext.plain_library_path()))
    lib.nab_workspace_bytes.restype = ctypes.c_int64
    assert lib.nab_workspace_bytes(8) > 0
    assert lib.nab_workspace_bytes(9) == -1
    for name in ("numa_all_reduce_init", "numa_all_reduce_dispose", "numa_all_reduce_register_buffer",
                 "numa_all_reduce_fp16", "numa_all_reduce_fp32", "numa_all_reduce_bf16", "nab_allreduce",
                 "nab_last_error", "nab_error_code", "nab_reset", "nab_set_auto_table", "nab_set_hybrid",
                 "nab_auto_protocol", "nab_reduce_scatter", "nab_all_gather"):
        assert hasattr(lib, name)
    buf = ctypes.create_string_buffer(256)
    assert lib.nab_last_error(buf, 256) > 0  # message of the failed call above
    assert b"world size" in buf.value
    assert lib.nab_reduce_scatter(None, None, None, None, ctypes.c_int64(8), 2) != 0
    lib.nab_last_error(buf, 256)
    assert b"null communicator" in buf.value
    assert lib.nab_all_gather(None, None, None, None, ctypes.c_int64(8), 2) != 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_c_abi_init_fails_cleanly_without_gpu():
    lib = ctypes.CDLL(str(_ext.plain_library_path()))
    lib.numa_all_reduce_init.restype = ctypes.c_void_p
    ptrs = (ctypes.c_void_p * 2)(4096, 8192)
    h = lib.numa_all_reduce_init(ptrs, None, 0, 0, 2, 1)
    assert h is None


def test_c_header_compiles_and_links(tmp_path):
    """A C program that includes nab_capi.h and nab_noalloc.h compiles as C11
    and links against libnab.so: the headers declare what the library
    exports."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    _ext.load()
    csrc = Path(_ext.plain_library_path()).parent / "csrc"
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    prog = tmp_path / "use_abi.c"
    prog.write_text(
        '#include "nab_capi.h"\n#include "nab_noalloc.h"\n#include <stdio.h>\n'
        "int main(void) {\n"
        "  char buf[128];\n"
        "  int64_t ws = nab_workspace_bytes(8);\n"
        "  int bad = nab_workspace_bytes(9) == -1 && nab_last_error(buf, sizeof buf) > 0;\n"
        "  void* fns[] = {(void*)numa_all_reduce_init, (void*)numa_all_reduce_dispose,\n"
        "    (void*)numa_all_reduce_register_buffer, (void*)numa_all_reduce_fp16, (void*)numa_all_reduce_fp32,\n"
        "    (void*)numa_all_reduce_bf16, (void*)nab_allreduce, (void*)nab_reduce_scatter, (void*)nab_all_gather,\n"
        "    (void*)nab_set_auto_table, (void*)nab_set_hybrid, (void*)nab_auto_protocol, (void*)nab_error_code,\n"
        "    (void*)nab_reset, (void*)nab_noalloc_emulated_allreduce, (void*)nab_noalloc_last_error};\n"
        "  for (unsigned i = 0; i < sizeof fns / sizeof fns[0]; ++i) if (!fns[i]) return 2;\n"
        '  printf("%lld %d\\n", (long long)ws, bad);\n'
        "  return ws > 0 && bad ? 0 : 1;\n}\n")
    lib = Path(_ext.plain_library_path())
    exe = tmp_path / "use_abi"
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", f"-I{csrc}", f"-I{cuda_inc}", str(prog), "-o", str(exe),
                    f"-L{lib.parent}", "-lnab", f"-Wl,-rpath,{lib.parent}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
