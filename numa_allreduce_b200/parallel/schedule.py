"""Pure-Python description of the allreduce schedules.

One description covers all three shapes of the algorithm, because each is the
hierarchical schedule for a particular grouping of the ranks:

* ``groups = [[0], [1], ..., [n-1]]``  -> one-shot: every rank owns the whole
  buffer and exchanges it with every other rank (stage 2 only);
* ``groups = [[0, 1, ..., n-1]]``      -> two-shot: reduce-scatter then
  all-gather inside one group (stages 1 and 3);
* ``groups = [[0, 1], [2, 3]]``        -> the reference's three-stage NUMA
  schedule: intra-group reduce-scatter, inter-group all-reduce of the
  partial sums between the owners of the same slice, intra-group all-gather.

This is the schedule the reference describes (docs/NUMA_ALLREDUCE_README.md
stage diagrams; dead kernels src/numa_all_reduce.cu:225-344) with its bugs
removed: every rank exchanges its slice with the same-slice owner of every
other group (not only "representatives"), stage 2 reads stage-1 results, and
stage 3 really gathers from peers.

The CPU emulator (:mod:`.emulate`) executes these objects over a gloo group,
the CUDA kernels implement the same arithmetic (fp32 accumulation in local
order, group partial sums kept in fp32 and added in group order, one
rounding to the input dtype at the end), and :func:`reference_allreduce`
computes the exact result both must give.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HierSchedule:
    groups: tuple[tuple[int, ...], ...]

    def __post_init__(self):
        if not self.groups or not all(self.groups):
            raise ValueError("groups must be non-empty")
        sizes = {len(g) for g in self.groups}
        if len(sizes) != 1:
            raise ValueError(f"all groups must have the same size, got {[len(g) for g in self.groups]}")
        flat = sorted(r for g in self.groups for r in g)
        if flat != list(range(len(flat))):
            raise ValueError(f"groups must partition ranks 0..{len(flat) - 1}: {self.groups}")

    # ---------------------------------------------------------- factories --
    @classmethod
    def from_groups(cls, groups) -> "HierSchedule":
        return cls(tuple(tuple(int(r) for r in g) for g in groups))

    @classmethod
    def oneshot(cls, world_size: int) -> "HierSchedule":
        return cls(tuple((r,) for r in range(world_size)))

    @classmethod
    def twoshot(cls, world_size: int) -> "HierSchedule":
        return cls((tuple(range(world_size)),))

    @classmethod
    def contiguous(cls, world_size: int, ngroups: int) -> "HierSchedule":
        """Contiguous groups, as the reference's build_numa_mappings
        (src/numa_all_reduce.cu:390-404)."""
        if world_size % ngroups:
            raise ValueError("world size must be divisible by the number of groups")
        per = world_size // ngroups
        return cls(tuple(tuple(range(g * per, (g + 1) * per)) for g in range(ngroups)))

    # ------------------------------------------------------------ queries --
    @property
    def world_size(self) -> int:
        return sum(len(g) for g in self.groups)

    @property
    def ngroups(self) -> int:
        return len(self.groups)

    @property
    def gsize(self) -> int:
        return len(self.groups[0])

    def group_of(self, rank: int) -> int:
        for gi, g in enumerate(self.groups):
            if rank in g:
                return gi
        raise ValueError(f"rank {rank} not in schedule")

    def local_index(self, rank: int) -> int:
        return self.groups[self.group_of(rank)].index(rank)

    def member(self, group: int, local: int) -> int:
        return self.groups[group][local]

    def slices(self, numel: int, align: int = 1) -> list[tuple[int, int]]:
        """Contiguous slice of each local index; boundaries are multiples of
        ``align`` elements (the last slice takes the remainder)."""
        n = self.gsize
        units = -(-numel // align)
        per = -(-units // n)
        out = []
        for i in range(n):
            a = min(numel, i * per * align)
            b = min(numel, (i + 1) * per * align)
            out.append((a, b))
        return out

    def stage1_peers(self, rank: int) -> list[int]:
        """Group members this rank exchanges reduce-scatter slices with."""
        g = self.group_of(rank)
        return [r for r in self.groups[g] if r != rank]

    def stage2_peers(self, rank: int) -> list[int]:
        """Owners of the same slice in the other groups."""
        g, l = self.group_of(rank), self.local_index(rank)
        return [self.member(h, l) for h in range(self.ngroups) if h != g]

    def stage3_peers(self, rank: int) -> list[int]:
        return self.stage1_peers(rank)

    def cross_group_bytes(self, nbytes: int) -> int:
        """Bytes each rank sends to other groups (stage 2): the traffic the
        reference's design minimises across NUMA sockets."""
        return (self.ngroups - 1) * -(-nbytes // self.gsize)


def reference_allreduce(inputs: list[torch.Tensor], schedule: HierSchedule) -> torch.Tensor:
    """Exact result of the schedule's arithmetic: per group, fp32 sum in local
    order; then fp32 sum of the group partials in group order; one rounding
    to the input dtype."""
    if len(inputs) != schedule.world_size:
        raise ValueError("one input per rank")
    dtype = inputs[0].dtype
    partials = []
    for g in schedule.groups:
        acc = inputs[g[0]].float().clone()
        for r in g[1:]:
            acc += inputs[r].float()
        partials.append(acc)
    acc = partials[0]
    for p in partials[1:]:
        acc = acc + p
    return acc.to(dtype)


def reference_reduce_scatter(inputs: list[torch.Tensor]) -> list[torch.Tensor]:
    """Exact result of the reduce-scatter collective: each input holds
    ``world_size`` equal segments (flattened); rank r gets the fp32 sum of
    segment r over the ranks in rank order, rounded once to the input dtype
    (the matching slice of the one-shot allreduce's result, bit for bit)."""
    ws = len(inputs)
    flat = [x.reshape(-1) for x in inputs]
    n = flat[0].numel()
    if n % ws or any(f.numel() != n for f in flat):
        raise ValueError("every input must hold world_size equal segments")
    seg = n // ws
    outs = []
    for r in range(ws):
        acc = flat[0][r * seg:(r + 1) * seg].float().clone()
        for q in range(1, ws):
            acc += flat[q][r * seg:(r + 1) * seg].float()
        outs.append(acc.to(inputs[0].dtype))
    return outs


def reference_all_gather(inputs: list[torch.Tensor]) -> torch.Tensor:
    """Exact result of the all-gather collective: the inputs in rank order."""
    return torch.cat([x.reshape(-1) for x in inputs])
