"""The native library builds for sm_100a and loads on a host without a GPU."""

import ctypes

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
