"""Fused tensor-parallel layer tail: allreduce + residual add + RMSNorm.

``fused_allreduce_rmsnorm`` runs one kernel that sums the row-parallel
partial outputs of all ranks over NVLink, adds the residual in place and
writes the RMSNorm of the new residual. ``rmsnorm_residual`` is the same
epilogue without communication (world size 1, and the norm of the unfused
baseline). Both are bf16 with fp32 accumulation.
"""

from __future__ import annotations

import torch

from . import _ext
from .allreduce import FUSED_ALGOS


def fused_allreduce_rmsnorm(comm, x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                            eps: float = 1e-5, algo: str = "auto", out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual += allreduce(x)``; returns ``rmsnorm(residual) * weight``.

    ``comm`` is a :class:`~numa_allreduce_b200.NumaAwareAllReduce`.
    """
    if comm.disabled:
        raise RuntimeError("communicator is disabled")
    if out is None:
        out = torch.empty_like(x)
    comm._ops.fused_ar_rmsnorm(comm._ptr, x, residual, weight, out, float(eps), FUSED_ALGOS[algo])
    return out


def rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual += x``; returns ``rmsnorm(residual) * weight`` (one kernel)."""
    ops = _ext.load()
    if out is None:
        out = torch.empty_like(x)
    ops.rmsnorm_residual(x, residual, weight, out, float(eps))
    return out


def reference_rmsnorm_residual(x_sum32: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                               eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 reference of the fused epilogue given the fp32 sum of partials:
    returns (new residual in bf16, normalised output in bf16)."""
    z = (x_sum32 + residual.float()).to(torch.bfloat16)
    zf = z.float()
    inv = torch.rsqrt(zf.pow(2).mean(dim=-1, keepdim=True) + eps)
    out = (zf * inv * weight.float()).to(torch.bfloat16)
    return z, out
