"""tcgen05 GEMM against a PyTorch fp32 reference of the same product."""

import pytest
import torch

from numa_allreduce_b200.ops.gemm import gemm, gemm_swiglu, interleave_gate_up, pack_weight

pytestmark = pytest.mark.gpu


def _rand(shape, seed, scale):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("T,N,K", [(1, 4096, 1792), (16, 4096, 1792), (7, 128, 64), (100, 256, 512),
                                   (128, 512, 1024), (512, 4096, 1792), (300, 384, 320)])
def test_gemm_matches_fp32(T, N, K):
    x = _rand((T, K), 1, 1.0)
    wt = _rand((N, K), 2, 0.02)
    y = gemm(x, wt, splits=1)
    ref = x.float() @ wt.float().t()
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,N,K,splits", [(1, 1280, 8192, 8), (8, 1024, 4096, 4), (32, 256, 1024, 2)])
def test_gemm_split_k(T, N, K, splits):
    x = _rand((T, K), 3, 1.0)
    wt = _rand((N, K), 4, 0.02)
    y = gemm(x, wt, splits=splits)
    ref = x.float() @ wt.float().t()
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_gemm_auto_splits_and_repeat():
    x = _rand((4, 8192), 5, 1.0)
    wt = _rand((1280, 8192), 6, 0.02)
    ref = x.float() @ wt.float().t()
    for _ in range(3):
        y = gemm(x, wt)
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_gemm_rejects_bad_shapes():
    x = _rand((4, 100), 7, 1.0)
    wt = _rand((128, 100), 8, 0.02)
    with pytest.raises((RuntimeError, ValueError)):
        gemm(x, wt)


def test_gemm_split_k_in_cuda_graph():
    """A split-K launch (one cluster per tile) replays exactly from a CUDA graph."""
    x = _rand((8, 3584), 9, 1.0)
    wt = _rand((8192, 3584), 10, 0.02)
    ref = x.float() @ wt.float().t()
    out = torch.empty(8, 8192, dtype=torch.bfloat16, device="cuda")
    gemm(x, wt, out=out, splits=4)  # first launch (attributes) outside capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gemm(x, wt, out=out, splits=4)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    del g


@pytest.mark.parametrize("T,N,K,splits", [(1, 1280, 8192, 0), (16, 512, 1024, 3), (200, 384, 640, 1)])
def test_gemm_packed_weight(T, N, K, splits):
    """The tiled weight layout gives the same product as the row-major one."""
    x = _rand((T, K), 11, 1.0)
    wt = _rand((N, K), 12, 0.02)
    pw = pack_weight(wt)
    assert torch.equal(pw.unpack(), wt)
    y = gemm(x, pw, splits=splits)
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), x.float() @ wt.float().t(), rtol=2e-2, atol=2e-2)
    assert torch.equal(y, gemm(x, wt, splits=splits))  # same split order, same bits


@pytest.mark.parametrize("T,I,K,splits,packed", [(1, 3584, 1024, 0, True), (16, 256, 512, 3, False),
                                                 (40, 128, 256, 1, True)])
def test_gemm_swiglu_epilogue(T, I, K, splits, packed):
    """silu(x @ gate.T) * (x @ up.T) from the interleaved gate|up weight."""
    x = _rand((T, K), 13, 1.0)
    wgu = _rand((2 * I, K), 14, 0.05)
    w = interleave_gate_up(wgu)
    y = gemm_swiglu(x, pack_weight(w) if packed else w, splits=splits)
    h = x.float() @ wgu.float().t()
    ref = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


def test_kernel_error_record_clean_after_good_launches():
    """GEMM and attention get the device's kernel error record; good
    launches leave it at zero (the wait path that writes it is exercised on
    the host in tests/test_kernel_errors_cpu.py)."""
    from numa_allreduce_b200 import check_kernels, reset_kernels
    from numa_allreduce_b200.ops import _ext

    reset_kernels()
    x = _rand((16, 1024), 7, 1.0)
    wt = _rand((512, 1024), 8, 0.02)
    gemm(x, wt)
    gemm_swiglu(x, interleave_gate_up(wt))
    ops = _ext.load()
    q = _rand((2, 8, 128), 9, 1.0)
    k = _rand((2, 1, 64, 128), 10, 1.0)
    v = _rand((2, 1, 64, 128), 11, 1.0)
    pos = torch.tensor([40], dtype=torch.int32, device="cuda")
    out = torch.empty(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    ops.decode_attention(q, k, v, pos, out, 2)
    torch.cuda.synchronize()
    check_kernels()
    assert list(ops.kernel_error_state()) == [0] * 8
