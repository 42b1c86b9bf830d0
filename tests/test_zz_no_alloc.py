"""The allocation-free C entry point matches the library's emulated two-shot.

``nab_noalloc_emulated_allreduce`` (exported by libnab.so) is for callers that
cannot call cudaMalloc where they reduce — code running while another
allocator holds all device memory, paths that must stay out of the driver's
allocator, or hosts that may not own device allocations. It keeps its scratch
in a static device array, so it is called here through its C symbol with only
inputs and outputs, twice in a row (the array keeps the previous call's
contents), and each result must equal, bit for bit (the tolerance of the
other allreduce tests), both the existing entry point's result and the CPU
fp32 rank-order sum. After each call its error record must read zero.

This file is collected last so that a failure here leaves every other test
already run.
"""

import ctypes

import pytest
import torch

from numa_allreduce_b200.ops import _ext
from numa_allreduce_b200.ops.allreduce import EmulatedGroup
from numa_allreduce_b200.parallel.schedule import HierSchedule, reference_allreduce

pytestmark = pytest.mark.gpu

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _library():
    _ext.load()  # builds libnab.so next to _C.so if needed
    return ctypes.CDLL(str(_ext.plain_library_path()))


def _entry_point():
    fn = _library().nab_noalloc_emulated_allreduce
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return fn


def _last_error():
    fn = _library().nab_noalloc_last_error
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    rec = (ctypes.c_uint32 * 8)()
    rc = fn(rec)
    return rc, list(rec)


def _call(fn, xs, outs):
    n = len(xs)
    ins = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
    ous = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return fn(ins, ous, n, xs[0].numel(), DTYPE_CODE[xs[0].dtype], stream)


@pytest.mark.parametrize("ws,dtype,numel", [(4, torch.bfloat16, 1 << 20), (8, torch.float32, 12345 * 4),
                                            (2, torch.float16, 8)])
def test_no_alloc_entry_point_matches_existing(ws, dtype, numel):
    torch.cuda.set_device(0)
    fn = _entry_point()
    with EmulatedGroup(ws) as g:
        for call in range(2):
            xs = [torch.randn(numel, device="cuda", generator=torch.Generator(device="cuda").manual_seed(
                10 * call + r)).to(dtype) for r in range(ws)]
            expected = g.all_reduce(xs, algo="twoshot")
            oracle = reference_allreduce([x.cpu() for x in xs], HierSchedule.twoshot(ws))
            outs = [torch.full_like(x, float("nan")) for x in xs]
            rc = _call(fn, xs, outs)
            torch.cuda.synchronize()
            assert rc == 0
            assert _last_error() == (0, [0] * 8), f"call {call}: a wait gave up"
            for r in range(ws):
                assert torch.equal(outs[r], expected[r]), f"call {call} rank {r}"
                assert torch.equal(outs[r].cpu(), oracle), f"call {call} rank {r} vs the CPU fp32 sum"


def test_no_alloc_rejects_bad_arguments():
    fn = _entry_point()
    xs = [torch.zeros(8, device="cuda") for _ in range(9)]
    assert _call(fn, xs[:9], xs[:9]) == 1  # more ranks than supported
    odd = [torch.zeros(3, device="cuda") for _ in range(2)]  # 12 bytes: not a multiple of 16
    assert _call(fn, odd, odd) == 1
