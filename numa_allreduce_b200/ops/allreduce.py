"""Thin wrappers over ``torch.ops.nab`` plus a single-GPU emulation group.

:class:`EmulatedGroup` runs the real multi-rank kernels for ``world_size``
ranks whose buffers all live on one GPU: each launch is ONE cooperative
kernel whose ``blockIdx.y`` selects the emulated rank, so CTAs that wait on
each other are guaranteed to be resident together. This is how the flag
protocols, the reduction order and the timeout path are tested on a single
B200 without separate launches waiting on one another.
"""

from __future__ import annotations

import torch

from ..utils.env import ALGO_IDS
from . import _ext

FUSED_ALGOS = {"auto": 0, "oneshot": 1, "twoshot": 2}


class EmulatedGroup:
    def __init__(self, world_size: int, device: torch.device | str = "cuda", *, oneshot_max: int = 1 << 20,
                 chunk_max: int = 0, max_ctas: int = 128, oneshot_ctas: int = 64,
                 fused_bytes: int = 512 << 10, timeout_ns: int = 2_000_000_000,
                 groups: list[list[int]] | None = None, pipe_ctas: int = 128, pipe_tile: int = 256 << 10):
        if not 2 <= world_size <= 8:
            raise ValueError("emulation needs 2..8 ranks")
        self.ops = _ext.load()
        self.world_size = world_size
        self.device = torch.device(device)
        cfg = [oneshot_max, chunk_max, max_ctas, oneshot_ctas, fused_bytes, timeout_ns, pipe_ctas, pipe_tile]
        lay = self.ops.layout(world_size, cfg)
        self.workspaces = [torch.zeros(int(lay[0]), dtype=torch.uint8, device=self.device)
                           for _ in range(world_size)]
        self.rank_data = [torch.empty(1 << 16, dtype=torch.uint8, device=self.device) for _ in range(world_size)]
        ptrs = [w.data_ptr() for w in self.workspaces]
        self.fas = [self.ops.init(ptrs, self.rank_data[r], r, True, cfg) for r in range(world_size)]
        if groups:
            flat = [r for g in groups for r in g]
            for fa in self.fas:
                self.ops.set_groups(fa, flat, len(groups))

    def all_reduce(self, inputs: list[torch.Tensor], algo: str = "twoshot",
                   outs: list[torch.Tensor] | None = None, participants: int = -1) -> list[torch.Tensor]:
        """One emulated allreduce. ``participants < world_size`` launches only
        the first ranks (the rest never arrive: used to test timeouts)."""
        outs = outs if outs is not None else [torch.empty_like(x) for x in inputs]
        self.ops.emulate_all_reduce(self.fas, inputs, outs, ALGO_IDS[algo], participants)
        return outs

    def reduce_scatter(self, inputs: list[torch.Tensor], outs: list[torch.Tensor] | None = None,
                       participants: int = -1) -> list[torch.Tensor]:
        """Emulated reduce-scatter: ``outs[r]`` = sum over ranks of segment r
        of ``inputs[q]`` (each input holds ``world_size`` equal segments)."""
        n = inputs[0].numel() // self.world_size
        outs = outs if outs is not None else [torch.empty(n, dtype=x.dtype, device=x.device) for x in inputs]
        self.ops.emulate_collective(self.fas, inputs, outs, 0, participants)
        return outs

    def all_gather(self, inputs: list[torch.Tensor], outs: list[torch.Tensor] | None = None,
                   participants: int = -1) -> list[torch.Tensor]:
        """Emulated all-gather: every ``outs[r]`` = the inputs in rank order."""
        n = inputs[0].numel() * self.world_size
        outs = outs if outs is not None else [torch.empty(n, dtype=x.dtype, device=x.device) for x in inputs]
        self.ops.emulate_collective(self.fas, inputs, outs, 1, participants)
        return outs

    def fused_ar_rmsnorm(self, inputs, residuals, weights, eps: float = 1e-5, algo: str = "auto",
                         outs=None):
        outs = outs if outs is not None else [torch.empty_like(x) for x in inputs]
        self.ops.emulate_fused_ar_rmsnorm(self.fas, inputs, residuals, weights, outs, eps, FUSED_ALGOS[algo])
        return outs

    def error_codes(self) -> list[int]:
        return [int(self.ops.error_code(fa)) for fa in self.fas]

    def error_states(self) -> list[list[int]]:
        return [list(self.ops.error_state(fa)) for fa in self.fas]

    def reset(self) -> None:
        torch.cuda.synchronize(self.device)
        for fa in self.fas:
            self.ops.reset(fa)

    def launches(self) -> int:
        return sum(int(self.ops.launches(fa)) for fa in self.fas)

    def close(self) -> None:
        for fa in self.fas:
            self.ops.dispose(fa)
        self.fas = []
        self.workspaces = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
