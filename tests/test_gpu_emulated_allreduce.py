"""Multi-rank allreduce kernels run for emulated ranks on ONE GPU.

Each launch is one cooperative kernel covering every emulated rank, so the
flag protocols, the reduction order and the double-buffering run exactly as
across GPUs. Results must equal the schedule's CPU oracle bit for bit
(fp32 accumulation in rank order, one rounding), which is stricter than the
reference's tolerance of 1e-2 for 16-bit types
(tests/test_numa_all_reduce.py:158-177).
"""

import pytest
import torch

from numa_allreduce_b200.ops.allreduce import EmulatedGroup
from numa_allreduce_b200.parallel.schedule import HierSchedule, reference_allreduce

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def _inputs(ws, numel, dtype, seed=0):
    out = []
    for r in range(ws):
        g = torch.Generator(device="cuda").manual_seed(seed * 100 + r)
        out.append(torch.randn(numel, generator=g, device="cuda", dtype=torch.float32).to(dtype))
    return out


def _schedule(algo, ws, groups=None):
    if algo == "oneshot":
        return HierSchedule.oneshot(ws)
    if algo in ("twoshot", "twoshot_pipe"):
        return HierSchedule.twoshot(ws)
    return HierSchedule.from_groups(groups)


@pytest.mark.parametrize("ws", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("algo", ["oneshot", "twoshot", "twoshot_pipe"])
def test_flat_protocols_bit_exact(ws, dtype, algo):
    per_pack = 16 // torch.tensor([], dtype=dtype).element_size()
    sizes = [per_pack, per_pack * 3, 1024, 4096 * 7 + per_pack * 5, 65536]
    if algo != "oneshot":
        sizes.append(1 << 21)  # several rounds per CTA at the emulation grid
    with EmulatedGroup(ws, chunk_max=16 << 10) as g:
        for n in sizes:
            xs = _inputs(ws, n, dtype, seed=n)
            outs = g.all_reduce(xs, algo=algo)
            torch.cuda.synchronize()
            assert g.error_codes() == [0] * ws
            ref = reference_allreduce([x.cpu() for x in xs], _schedule(algo, ws))
            for r in range(ws):
                assert torch.equal(outs[r].cpu(), ref), f"rank {r} size {n}"


@pytest.mark.parametrize("groups", [[[0, 1], [2, 3]], [[0, 2], [1, 3]], [[0, 1, 2, 3], [4, 5, 6, 7]],
                                    [[0, 1], [2, 3], [4, 5], [6, 7]]])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_hierarchical_bit_exact(groups, dtype):
    ws = sum(len(x) for x in groups)
    with EmulatedGroup(ws, chunk_max=16 << 10, groups=groups) as g:
        for n in [8, 4096 + 8, 1 << 20]:
            xs = _inputs(ws, n, dtype, seed=n + 1)
            outs = g.all_reduce(xs, algo="hier")
            torch.cuda.synchronize()
            assert g.error_codes() == [0] * ws
            ref = reference_allreduce([x.cpu() for x in xs], HierSchedule.from_groups(groups))
            for r in range(ws):
                assert torch.equal(outs[r].cpu(), ref)


def test_hier_matches_numa_config_tolerance():
    """Hierarchical shape (2 groups of 4, bf16 1 MB) against an fp32 sum."""
    groups = [[0, 1, 2, 3], [4, 5, 6, 7]]
    with EmulatedGroup(8, groups=groups) as g:
        xs = _inputs(8, (1 << 20) // 2, torch.bfloat16, seed=7)
        outs = g.all_reduce(xs, algo="hier")
        exact = torch.stack([x.float() for x in xs]).sum(0)
        torch.testing.assert_close(outs[3].float(), exact, rtol=1e-2, atol=1e-2)


def test_back_to_back_calls_and_protocol_switches():
    """Epochs and double buffers across many calls with changing grids."""
    ws = 4
    with EmulatedGroup(ws, chunk_max=16 << 10, groups=[[0, 1], [2, 3]]) as g:
        algos = ["oneshot", "twoshot", "hier", "twoshot_pipe"]
        for i in range(1200):
            n = [8, 1000 * 8, 50000 * 8, 8 * 3][i % 4]
            algo = algos[i % 4]
            xs = _inputs(ws, n, torch.bfloat16, seed=i)
            outs = g.all_reduce(xs, algo=algo)
            if i % 50 == 0 or i > 1190:
                sched = {"oneshot": HierSchedule.oneshot(ws), "twoshot": HierSchedule.twoshot(ws),
                         "twoshot_pipe": HierSchedule.twoshot(ws),
                         "hier": HierSchedule.from_groups([[0, 1], [2, 3]])}[algo]
                ref = reference_allreduce([x.cpu() for x in xs], sched)
                for r in range(ws):
                    assert torch.equal(outs[r].cpu(), ref), (i, algo)
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws


def test_in_place():
    ws = 4
    with EmulatedGroup(ws) as g:
        for algo, n in [("oneshot", 4096), ("twoshot", 1 << 20), ("twoshot_pipe", 3 << 20)]:
            xs = _inputs(ws, n, torch.bfloat16, seed=3)
            ref = reference_allreduce([x.cpu() for x in xs], _schedule(algo, ws))
            g.all_reduce(xs, algo=algo, outs=xs)
            for r in range(ws):
                assert torch.equal(xs[r].cpu(), ref)


@pytest.mark.parametrize("algo", ["oneshot", "twoshot", "hier", "twoshot_pipe"])
def test_absent_rank_times_out_and_recovers(algo):
    """A rank that never launches: the others' bounded waits give up, the
    error word names the stage, the context stays usable, and after reset()
    the group works again."""
    ws = 4
    groups = [[0, 1], [2, 3]]
    with EmulatedGroup(ws, timeout_ns=200_000_000, groups=groups) as g:
        xs = _inputs(ws, 1 << 16, torch.float32)
        g.all_reduce(xs, algo=algo, participants=ws - 1)
        torch.cuda.synchronize()  # returns: nothing hangs
        codes = g.error_codes()
        assert codes[0] == 1  # kErrTimeout (emulated launches report on rank 0's record)
        state = g.error_states()[0]
        assert state[7] >= 1  # at least one wait gave up
        g.reset()
        assert g.error_codes() == [0] * ws
        outs = g.all_reduce(xs, algo=algo)
        torch.cuda.synchronize()
        ref = reference_allreduce([x.cpu() for x in xs],
                                  _schedule(algo, ws, groups) if algo != "hier" else HierSchedule.from_groups(groups))
        assert torch.equal(outs[1].cpu(), ref)


def test_bad_arguments_raise():
    with EmulatedGroup(2) as g:
        x = [torch.zeros(12, device="cuda", dtype=torch.float32) for _ in range(2)]  # 48 B: fine
        g.all_reduce(x, algo="oneshot")
        bad = [torch.zeros(3, device="cuda", dtype=torch.float32) for _ in range(2)]  # 12 B
        with pytest.raises((RuntimeError, ValueError)):
            g.all_reduce(bad, algo="oneshot")
        big = [torch.zeros((2 << 20) // 4, device="cuda") for _ in range(2)]  # beyond one-shot slot
        with pytest.raises((RuntimeError, ValueError)):
            g.all_reduce(big, algo="oneshot")
        with pytest.raises((RuntimeError, ValueError)):
            g.all_reduce(x, algo="hier")  # no groups set
