"""tcgen05 GEMM for the tensor-parallel projections, and its fusion with the
allreduce + residual + RMSNorm of a row-parallel layer.

Weights are stored K-major (``wt`` is ``[out_features, in_features]``, the
layout of ``torch.nn.Linear.weight``), so ``gemm(x, wt) == x @ wt.T``.
"""

from __future__ import annotations

import torch

from . import _ext
from .errors import after_launch

TILE_N, TILE_K = 128, 64


class PackedWeight:
    """A ``[N, K]`` bf16 weight re-laid as ``[N/128][K/64]`` tiles of 128 x 64,
    each tile 16 KB of contiguous memory: every weight load of the GEMM then
    reads one contiguous block of HBM instead of 128 rows ``2K`` bytes apart.
    Built once, at weight-load time, by :func:`pack_weight`."""

    def __init__(self, data: torch.Tensor, n: int, k: int):
        self.data, self.n, self.k = data, n, k

    @property
    def shape(self):
        return (self.n, self.k)

    def numel(self) -> int:
        return self.n * self.k

    def unpack(self) -> torch.Tensor:
        return (self.data.view(self.n // TILE_N, self.k // TILE_K, TILE_N, TILE_K)
                .permute(0, 2, 1, 3).reshape(self.n, self.k))


def pack_weight(wt: torch.Tensor) -> PackedWeight:
    n, k = wt.shape
    if n % TILE_N or k % TILE_K:
        raise ValueError("pack_weight needs N % 128 == 0 and K % 64 == 0")
    data = wt.view(n // TILE_N, TILE_N, k // TILE_K, TILE_K).permute(0, 2, 1, 3).reshape(n * k // TILE_K, TILE_K)
    return PackedWeight(data.contiguous(), n, k)


def interleave_gate_up(wgu: torch.Tensor) -> torch.Tensor:
    """``[2I, K]`` gate|up rows (gate rows first) -> 64-row blocks alternating
    gate and up, so that every 128-row tile holds the gate and up rows of the
    same 64 features (the layout :func:`gemm_swiglu` reads)."""
    two_i, k = wgu.shape
    i = two_i // 2
    if two_i % 2 or i % 64:
        raise ValueError("interleave_gate_up needs an intermediate size that is a multiple of 64")
    return wgu.view(2, i // 64, 64, k).permute(1, 0, 2, 3).reshape(two_i, k).contiguous()


def _operand(wt):
    return (wt.data, wt.n, True) if isinstance(wt, PackedWeight) else (wt, wt.shape[0], False)


def gemm(x: torch.Tensor, wt, out: torch.Tensor | None = None, splits: int | None = None) -> torch.Tensor:
    """``x[T, K] @ wt[N, K].T`` in bf16 with fp32 accumulation (N % 128 == 0, K % 64 == 0).

    ``wt`` is a ``[N, K]`` tensor or a :class:`PackedWeight`. ``splits`` CTAs
    share each output tile's K loop (one thread-block cluster, partials added
    over distributed shared memory); ``None`` picks the count."""
    ops = _ext.load()
    data, N, packed = _operand(wt)
    if out is None:
        out = torch.empty(x.shape[0], N, dtype=torch.bfloat16, device=x.device)
    ops.gemm(x, data, out, int(splits or 0), packed, False)
    after_launch()
    return out


def gemm_swiglu(x: torch.Tensor, wgu, out: torch.Tensor | None = None, splits: int | None = None) -> torch.Tensor:
    """SwiGLU projection in one launch: ``silu(x @ gate.T) * (x @ up.T)``.

    ``wgu`` is the gate|up weight re-laid by :func:`interleave_gate_up`
    (a tensor or its :class:`PackedWeight`); the epilogue applies the
    activation to the fp32 accumulators and writes ``[T, I]``."""
    ops = _ext.load()
    data, N, packed = _operand(wgu)
    if out is None:
        out = torch.empty(x.shape[0], N // 2, dtype=torch.bfloat16, device=x.device)
    ops.gemm(x, data, out, int(splits or 0), packed, True)
    after_launch()
    return out


GEMM_AR_MODES = {"auto": 0, "oneshot": 1, "reduce_scatter": 2}


def gemm_allreduce_rmsnorm(comm, x: torch.Tensor, wt: torch.Tensor, residual: torch.Tensor,
                           weight: torch.Tensor, eps: float = 1e-5, out: torch.Tensor | None = None,
                           splits: int = 0, mode: str = "auto") -> torch.Tensor:
    """Row-parallel layer tail: ``residual += allreduce(x @ wt.T)``; returns
    ``rmsnorm(residual) * weight``, in two launches.

    ``mode="oneshot"``: the GEMM's epilogue stores each finished bf16 output
    tile into every rank's buffer over NVLink and raises a flag per tile; the
    second launch waits for the tiles, sums the ranks in rank order, adds the
    residual and normalises. ``mode="reduce_scatter"``: the epilogue stores
    token row ``t`` only into rank ``t % world_size``; the second launch
    reduces the rows this rank owns, applies residual + norm, and gathers the
    other owners' new residual rows (about 2/ws of the one-shot's NVLink
    bytes, one more flag exchange). ``"auto"`` takes the reduce-scatter from
    4 ranks and 256 rows on (at 2 ranks both move the same bytes). ``splits=0`` picks the split-K factor (split partials
    are added on this GPU before the tile is sent)."""
    if out is None:
        out = torch.empty_like(residual)
    data, _, packed = _operand(wt)
    comm._ops.gemm_ar_rmsnorm(comm._ptr, x, data, residual, weight, out, float(eps), int(splits), packed,
                              GEMM_AR_MODES[mode])
    if comm.env.check and not torch.cuda.is_current_stream_capturing():
        torch.cuda.current_stream().synchronize()
        comm.check()
    return out
