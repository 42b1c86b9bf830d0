"""CPU executor of :class:`HierSchedule` over a torch.distributed group.

Runs the three stages with point-to-point sends and receives (gloo on CPU),
so the schedule's plumbing (who sends which slice to whom, in which order the
partial sums are added) is tested without a GPU. The result equals
:func:`~numa_allreduce_b200.parallel.schedule.reference_allreduce` bit for bit
and ``dist.all_reduce(SUM)`` to rounding.

:func:`emulate_reduce_scatter` and :func:`emulate_all_gather` execute the
contiguous-segment collectives the same way (segment j to its owner j, owner
adds in rank order; own segment to every peer, concatenation in rank order).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .schedule import HierSchedule


def _global(group, r: int) -> int:
    return r if group is None else dist.get_global_rank(group, r)


def _exchange(send: dict[int, torch.Tensor], recv_shapes: dict[int, tuple[int, torch.dtype]],
              group) -> dict[int, torch.Tensor]:
    """Sends ``send[peer]`` to each peer and receives one tensor from each peer
    in ``recv_shapes``. Tensors travel as raw bytes, so any dtype works."""
    ops = []
    recv = {}
    for peer, (numel, dtype) in sorted(recv_shapes.items()):
        buf = torch.empty(numel, dtype=dtype)
        recv[peer] = buf
        if numel:
            ops.append(dist.P2POp(dist.irecv, buf.view(torch.uint8), _global(group, peer), group))
    for peer, t in sorted(send.items()):
        if t.numel():
            ops.append(dist.P2POp(dist.isend, t.contiguous().view(torch.uint8), _global(group, peer), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return recv


def emulate_allreduce(tensor: torch.Tensor, schedule: HierSchedule, group=None) -> torch.Tensor:
    """Allreduce (SUM) of ``tensor`` across the ranks of ``group`` following
    ``schedule``. Every rank must call it with the same shape and dtype."""
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    if ws != schedule.world_size:
        raise ValueError(f"schedule is for {schedule.world_size} ranks, group has {ws}")
    dtype = tensor.dtype
    x = tensor.detach().reshape(-1).cpu().contiguous()
    sl = schedule.slices(x.numel())
    g, l = schedule.group_of(rank), schedule.local_index(rank)
    a, b = sl[l]

    # stage 1: intra-group reduce-scatter (slice m goes to local index m)
    peers1 = schedule.stage1_peers(rank)
    send1 = {p: x[sl[schedule.local_index(p)][0]:sl[schedule.local_index(p)][1]] for p in peers1}
    recv1 = _exchange(send1, {p: (b - a, dtype) for p in peers1}, group)
    acc = None
    for m, member in enumerate(schedule.groups[g]):
        part = x[a:b] if member == rank else recv1[member]
        acc = part.float().clone() if acc is None else acc + part.float()
    partial = acc  # fp32: the only rounding happens after stage 2

    # stage 2: same-slice owners of the other groups exchange fp32 partial sums
    peers2 = schedule.stage2_peers(rank)
    recv2 = _exchange({p: partial for p in peers2}, {p: (b - a, torch.float32) for p in peers2}, group)
    acc = None
    for h in range(schedule.ngroups):
        owner = schedule.member(h, l)
        part = partial if owner == rank else recv2[owner]
        acc = part.clone() if acc is None else acc + part
    final = acc.to(dtype)

    # stage 3: intra-group all-gather
    out = torch.empty_like(x)
    out[a:b] = final
    peers3 = schedule.stage3_peers(rank)
    shapes = {p: (sl[schedule.local_index(p)][1] - sl[schedule.local_index(p)][0], dtype) for p in peers3}
    recv3 = _exchange({p: final for p in peers3}, shapes, group)
    for p, t in recv3.items():
        pa, pb = sl[schedule.local_index(p)]
        out[pa:pb] = t
    return out.view(tensor.shape).to(tensor.device)


def emulate_reduce_scatter(tensor: torch.Tensor, group=None) -> torch.Tensor:
    """Reduce-scatter (SUM) over ``group``: ``tensor`` holds world_size equal
    segments; this rank gets the sum of segment ``rank``, accumulated in fp32
    in rank order and rounded once."""
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    x = tensor.detach().reshape(-1).cpu().contiguous()
    if x.numel() % ws:
        raise ValueError("the input must hold world_size equal segments")
    seg = x.numel() // ws
    peers = [p for p in range(ws) if p != rank]
    recv = _exchange({p: x[p * seg:(p + 1) * seg] for p in peers}, {p: (seg, x.dtype) for p in peers}, group)
    acc = None
    for q in range(ws):
        part = x[rank * seg:(rank + 1) * seg] if q == rank else recv[q]
        acc = part.float().clone() if acc is None else acc + part.float()
    return acc.to(tensor.dtype).to(tensor.device)


def emulate_all_gather(tensor: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather over ``group``: every rank's ``tensor`` (flattened) in rank
    order."""
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    x = tensor.detach().reshape(-1).cpu().contiguous()
    peers = [p for p in range(ws) if p != rank]
    recv = _exchange({p: x for p in peers}, {p: (x.numel(), x.dtype) for p in peers}, group)
    parts = [x if q == rank else recv[q] for q in range(ws)]
    return torch.cat(parts).to(tensor.device)
