"""Weight layouts read by the tcgen05 GEMM (pure tensor reshapes, checked on
the CPU): the tiled layout of pack_weight and the gate/up interleave of the
SwiGLU epilogue."""

import pytest
import torch

from numa_allreduce_b200.ops.gemm import TILE_K, TILE_N, interleave_gate_up, pack_weight


def test_pack_weight_tiles_are_contiguous_and_round_trip():
    n, k = 256, 192
    w = torch.arange(n * k, dtype=torch.float32).reshape(n, k).to(torch.bfloat16)
    pw = pack_weight(w)
    assert pw.shape == (n, k) and pw.numel() == n * k
    assert pw.data.shape == (n * k // TILE_K, TILE_K) and pw.data.is_contiguous()
    # tile (m, kb) is rows [(m * K/64 + kb) * 128, +128) of the packed matrix
    kbt = k // TILE_K
    for m in range(n // TILE_N):
        for kb in range(kbt):
            tile = pw.data[(m * kbt + kb) * TILE_N:(m * kbt + kb + 1) * TILE_N]
            assert torch.equal(tile, w[m * TILE_N:(m + 1) * TILE_N, kb * TILE_K:(kb + 1) * TILE_K])
    assert torch.equal(pw.unpack(), w)


@pytest.mark.parametrize("shape", [(100, 64), (128, 100), (129, 64)])
def test_pack_weight_rejects_untileable_shapes(shape):
    with pytest.raises(ValueError):
        pack_weight(torch.zeros(shape, dtype=torch.bfloat16))


def test_interleave_gate_up_blocks():
    i, k = 192, 8
    gate = torch.arange(i * k, dtype=torch.float32).reshape(i, k)
    up = -gate
    w = interleave_gate_up(torch.cat([gate, up]))
    for j in range(i // 64):
        assert torch.equal(w[128 * j:128 * j + 64], gate[64 * j:64 * (j + 1)])
        assert torch.equal(w[128 * j + 64:128 * (j + 1)], up[64 * j:64 * (j + 1)])


def test_interleave_gate_up_rejects_bad_sizes():
    with pytest.raises(ValueError):
        interleave_gate_up(torch.zeros(2 * 100, 8))
