"""Schedules and their gloo/CPU executor (the 3-stage hierarchical emulation on
gloo ranks, fp32 [1024, 1024]).

Config 1: world size 4 over gloo, the three-stage schedule with NUMA groups
{0,1},{2,3}; each rank holds fp32 [1024, 1024] drawn from N(0,1) with
seed=rank; the result must equal dist.all_reduce(SUM) within 1e-5 abs, and
topology detection runs on the host in every rank.
"""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from numa_allreduce_b200.parallel.emulate import emulate_allreduce
from numa_allreduce_b200.parallel.schedule import HierSchedule, reference_allreduce


def test_schedule_validation():
    with pytest.raises(ValueError):
        HierSchedule.from_groups([[0, 1], [2]])
    with pytest.raises(ValueError):
        HierSchedule.from_groups([[0, 1], [1, 2]])
    s = HierSchedule.from_groups([[0, 2], [1, 3]])
    assert s.world_size == 4 and s.gsize == 2 and s.ngroups == 2
    assert s.group_of(2) == 0 and s.local_index(3) == 1
    assert s.stage1_peers(0) == [2] and s.stage2_peers(0) == [1]
    assert HierSchedule.contiguous(8, 2).groups == ((0, 1, 2, 3), (4, 5, 6, 7))
    assert HierSchedule.oneshot(3).stage2_peers(1) == [0, 2]
    assert HierSchedule.twoshot(3).stage2_peers(1) == []


def test_slices_cover_everything():
    s = HierSchedule.twoshot(3)
    for n in [0, 1, 7, 8, 1000, 1001]:
        sl = s.slices(n, align=8)
        assert sl[0][0] == 0 and sl[-1][1] == n
        assert all(a <= b for a, b in sl)
        assert all(sl[i][1] == sl[i + 1][0] for i in range(len(sl) - 1))


def test_cross_group_traffic():
    """The reference's design goal: stage 2 moves 1/g of the data across groups."""
    s = HierSchedule.contiguous(8, 2)
    assert s.cross_group_bytes(1 << 20) == (1 << 20) // 4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_reference_allreduce_variants(dtype):
    xs = [torch.randn(4096, generator=torch.Generator().manual_seed(r)).to(dtype) for r in range(4)]
    exact = torch.stack([x.double() for x in xs]).sum(0)
    for s in (HierSchedule.oneshot(4), HierSchedule.twoshot(4), HierSchedule.contiguous(4, 2)):
        out = reference_allreduce(xs, s)
        assert out.dtype == dtype
        tol = 1e-5 if dtype == torch.float32 else 2e-2
        torch.testing.assert_close(out.double(), exact, rtol=tol, atol=tol)
    # flat one-shot and two-shot round once: identical results
    assert torch.equal(reference_allreduce(xs, HierSchedule.oneshot(4)),
                       reference_allreduce(xs, HierSchedule.twoshot(4)))


def _worker(rank, ws, port, groups, dtype_name, shape, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from numa_allreduce_b200 import detect_numa_topology

        topo = detect_numa_topology()
        assert len(topo.numa_nodes) >= 1
        dtype = getattr(torch, dtype_name)
        torch.manual_seed(rank)
        x = torch.randn(shape, dtype=torch.float32).to(dtype)
        expected = x.clone().float()
        dist.all_reduce(expected)
        sched = HierSchedule.from_groups(groups)
        out = emulate_allreduce(x, sched, group=None)
        everyone = [torch.empty(x.shape) for _ in range(ws)]
        dist.all_gather(everyone, x.float())  # gloo gathers fp32; the round trip is exact
        exact = reference_allreduce([e.to(dtype) for e in everyone], sched)
        err = (out.float() - expected).abs().max().item()
        result_q.put((rank, err, torch.equal(out, exact), tuple(out.shape)))
    finally:
        dist.destroy_process_group()


def _run(ws, groups, dtype_name, shape):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker, args=(ws, free_port(), groups, dtype_name, shape, q), nprocs=ws, join=True)
    return [q.get() for _ in range(ws)]


def test_baseline_config1_three_stage_gloo():
    res = _run(4, [[0, 1], [2, 3]], "float32", (1024, 1024))
    for rank, err, exact, shape in res:
        assert shape == (1024, 1024)
        assert err <= 1e-5, f"rank {rank}: max abs error {err}"
        assert exact


@pytest.mark.parametrize("groups", [[[0], [1], [2]], [[0, 1, 2]]])
def test_flat_schedules_gloo(groups):
    res = _run(3, groups, "bfloat16", (4097,))
    for rank, err, exact, _ in res:
        assert exact
        assert err <= 0.05
