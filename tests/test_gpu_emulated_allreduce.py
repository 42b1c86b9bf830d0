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
from numa_allreduce_b200.parallel.schedule import (HierSchedule, reference_all_gather, reference_allreduce,
                                                   reference_reduce_scatter)

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


@pytest.mark.parametrize("ws", [2, 3, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
def test_reduce_scatter_and_all_gather_bit_exact(ws, dtype):
    """Segment collectives against the CPU oracle; segments longer than the
    one-shot slot (64 KiB here) run as several launches, piece by piece."""
    per_pack = 16 // torch.tensor([], dtype=dtype).element_size()
    esz = torch.tensor([], dtype=dtype).element_size()
    with EmulatedGroup(ws, oneshot_max=64 << 10) as g:
        for seg in [per_pack, per_pack * 5, 4096 + per_pack * 3, (64 << 10) // esz, (200 << 10) // esz + per_pack]:
            xs = _inputs(ws, ws * seg, dtype, seed=seg)
            before = g.launches()
            outs = g.reduce_scatter(xs)
            torch.cuda.synchronize()
            assert g.error_codes() == [0] * ws
            pieces = -(-seg * esz // (64 << 10))
            assert g.launches() - before == pieces * ws
            ref = reference_reduce_scatter([x.cpu() for x in xs])
            for r in range(ws):
                assert torch.equal(outs[r].cpu(), ref[r]), f"reduce-scatter rank {r} segment {seg}"
            mine = [x[:seg].contiguous() for x in xs]
            gathered = g.all_gather(mine)
            torch.cuda.synchronize()
            assert g.error_codes() == [0] * ws
            ref = reference_all_gather([m.cpu() for m in mine])
            for r in range(ws):
                assert torch.equal(gathered[r].cpu(), ref), f"all-gather rank {r} segment {seg}"


def test_reduce_scatter_matches_allreduce_slice():
    """Same arithmetic as the allreduce: bit-identical to its slice."""
    ws = 4
    with EmulatedGroup(ws) as g:
        xs = _inputs(ws, ws * 8192, torch.bfloat16, seed=5)
        full = g.all_reduce(xs, algo="oneshot")
        parts = g.reduce_scatter(xs)
        torch.cuda.synchronize()
        for r in range(ws):
            assert torch.equal(parts[r], full[0][r * 8192:(r + 1) * 8192])


def test_collectives_interleaved_with_allreduce():
    """Epochs and the shared one-shot slots across mixed call types."""
    ws = 4
    with EmulatedGroup(ws, chunk_max=16 << 10) as g:
        for i in range(300):
            n = [64, 4000 * 8, 8][i % 3]
            xs = _inputs(ws, ws * n, torch.float16, seed=i)
            kind = i % 3
            if kind == 0:
                outs = g.all_reduce(xs, algo=["oneshot", "twoshot", "twoshot_pipe"][i % 3 + (i // 3) % 2])
                ref = reference_allreduce([x.cpu() for x in xs], HierSchedule.oneshot(ws))
                if i % 30 == 0:
                    assert all(torch.equal(o.cpu(), ref) for o in outs), i
            elif kind == 1:
                outs = g.reduce_scatter(xs)
                if i % 30 == 1:
                    ref = reference_reduce_scatter([x.cpu() for x in xs])
                    assert all(torch.equal(outs[r].cpu(), ref[r]) for r in range(ws)), i
            else:
                mine = [x[:n].contiguous() for x in xs]
                outs = g.all_gather(mine)
                if i % 30 == 2:
                    ref = reference_all_gather([m.cpu() for m in mine])
                    assert all(torch.equal(o.cpu(), ref) for o in outs), i
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws


@pytest.mark.parametrize("kind", ["reduce_scatter", "all_gather"])
def test_collective_absent_rank_times_out_and_recovers(kind):
    ws = 4
    with EmulatedGroup(ws, timeout_ns=200_000_000) as g:
        xs = _inputs(ws, ws * 4096, torch.float32)
        fn = getattr(g, kind)
        args = xs if kind == "reduce_scatter" else [x[:4096].contiguous() for x in xs]
        fn(args, participants=ws - 1)
        torch.cuda.synchronize()  # returns: nothing hangs
        assert g.error_codes()[0] == 1  # kErrTimeout
        state = g.error_states()[0]
        assert state[3] == (14 if kind == "reduce_scatter" else 15)  # the collective's stage tag
        g.reset()
        outs = fn(args)
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws
        if kind == "reduce_scatter":
            assert torch.equal(outs[2].cpu(), reference_reduce_scatter([x.cpu() for x in xs])[2])
        else:
            assert torch.equal(outs[1].cpu(), reference_all_gather([a.cpu() for a in args]))


def test_collective_bad_arguments_raise():
    with EmulatedGroup(2) as g:
        xs = [torch.zeros(2 * 12, device="cuda") for _ in range(2)]
        g.reduce_scatter(xs)
        with pytest.raises((RuntimeError, ValueError)):
            g.reduce_scatter([torch.zeros(2 * 3, device="cuda") for _ in range(2)])  # 12-byte segments
        with pytest.raises((RuntimeError, ValueError)):
            g.all_gather([torch.zeros(8, device="cuda") for _ in range(2)],
                         outs=[torch.zeros(8, device="cuda") for _ in range(2)])  # output too small
        with pytest.raises((RuntimeError, ValueError)):
            g.reduce_scatter(xs, outs=[x[:12] for x in xs])  # output aliases the input
