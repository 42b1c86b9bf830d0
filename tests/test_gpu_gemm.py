"""tcgen05 GEMM against a PyTorch fp32 reference of the same product."""

import pytest
import torch

from numa_allreduce_b200.ops.gemm import gemm

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
