"""Fused allreduce + residual add + RMSNorm against a PyTorch fp32 reference."""

import pytest
import torch

from numa_allreduce_b200.ops.allreduce import EmulatedGroup
from numa_allreduce_b200.ops.fused import reference_rmsnorm_residual, rmsnorm_residual

pytestmark = pytest.mark.gpu


def _seqsum(xs):
    """fp32 sum in rank order (the kernels' order)."""
    acc = xs[0].float().clone()
    for x in xs[1:]:
        acc += x.float()
    return acc


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("T,H", [(1, 4096), (7, 4096), (64, 8192), (3, 128)])
def test_rmsnorm_residual_local(T, H):
    x = _rand((T, H), 1)
    res = _rand((T, H), 2)
    w = _rand((H,), 3) + 1
    res_in = res.clone()
    out = rmsnorm_residual(x, res, w, eps=1e-5)
    ref_res, ref_out = reference_rmsnorm_residual(x.float(), res_in, w, 1e-5)
    assert torch.equal(res, ref_res)
    torch.testing.assert_close(out.float(), ref_out.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("ws", [2, 4, 8])
@pytest.mark.parametrize("algo", ["oneshot", "twoshot"])
@pytest.mark.parametrize("T,H", [(1, 4096), (5, 8192), (16, 4096), (37, 1024)])
def test_fused_emulated(ws, algo, T, H):
    if algo == "oneshot" and T * H * 2 > (512 << 10):
        pytest.skip("beyond the one-shot slot")
    with EmulatedGroup(ws) as g:
        xs = [_rand((T, H), 10 + r, 0.5) for r in range(ws)]
        res = _rand((T, H), 99)
        w = _rand((H,), 98) + 1
        residuals = [res.clone() for _ in range(ws)]
        weights = [w.clone() for _ in range(ws)]
        outs = g.fused_ar_rmsnorm(xs, residuals, weights, eps=1e-5, algo=algo)
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws
        s32 = _seqsum(xs)
        ref_res, ref_out = reference_rmsnorm_residual(s32, res, w, 1e-5)
        for r in range(ws):
            assert torch.equal(residuals[r], ref_res), f"rank {r} residual"
            torch.testing.assert_close(outs[r].float(), ref_out.float(), rtol=1e-2, atol=1e-2)
            # every rank holds the same bits
            assert torch.equal(outs[r], outs[0])


def test_fused_repeated_calls():
    ws, T, H = 4, 24, 4096
    with EmulatedGroup(ws) as g:
        w = _rand((H,), 5) + 1
        for i in range(50):
            algo = ["oneshot", "twoshot"][i % 2]
            xs = [_rand((T, H), 1000 * i + r, 0.5) for r in range(ws)]
            res = _rand((T, H), i)
            residuals = [res.clone() for _ in range(ws)]
            outs = g.fused_ar_rmsnorm(xs, residuals, [w] * ws, algo=algo)
            if i % 10 == 9:
                s32 = _seqsum(xs)
                ref_res, ref_out = reference_rmsnorm_residual(s32, res, w, 1e-5)
                assert torch.equal(residuals[2], ref_res)
                torch.testing.assert_close(outs[1].float(), ref_out.float(), rtol=1e-2, atol=1e-2)
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws
