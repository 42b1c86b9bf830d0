"""tcgen05 GEMM for the tensor-parallel projections, and its fusion with the
allreduce + residual + RMSNorm of a row-parallel layer.

Weights are stored K-major (``wt`` is ``[out_features, in_features]``, the
layout of ``torch.nn.Linear.weight``), so ``gemm(x, wt) == x @ wt.T``.
"""

from __future__ import annotations

import torch

from . import _ext


def gemm(x: torch.Tensor, wt: torch.Tensor, out: torch.Tensor | None = None,
         splits: int | None = None) -> torch.Tensor:
    """``x[T, K] @ wt[N, K].T`` in bf16 with fp32 accumulation (N % 128 == 0, K % 64 == 0)."""
    ops = _ext.load()
    T, K = x.shape
    N = wt.shape[0]
    if out is None:
        out = torch.empty(T, N, dtype=torch.bfloat16, device=x.device)
    if splits is None:
        splits = int(ops.gemm_splits(T, N, K))
    ws = torch.empty(splits * T * N, dtype=torch.float32, device=x.device) if splits > 1 else None
    ops.gemm(x, wt, out, ws, splits)
    return out


def gemm_allreduce_rmsnorm(comm, x: torch.Tensor, wt: torch.Tensor, residual: torch.Tensor,
                           weight: torch.Tensor, eps: float = 1e-5, out: torch.Tensor | None = None,
                           splits: int = 0) -> torch.Tensor:
    """Row-parallel layer tail: ``residual += allreduce(x @ wt.T)``; returns
    ``rmsnorm(residual) * weight``. The GEMM's epilogue stores each partial
    tile into every rank's buffer over NVLink; a second launch sums them.
    ``splits=0`` picks the split-K factor (fp32 partials when > 1)."""
    if out is None:
        out = torch.empty_like(residual)
    comm._ops.gemm_ar_rmsnorm(comm._ptr, x, wt, residual, weight, out, float(eps), int(splits))
    return out
