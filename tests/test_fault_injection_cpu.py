"""Failure detection without a GPU fault: failures are made on the host.

* heartbeat monitor (PeerMonitor): a rank that stops beating is reported dead
  within the timeout, a rank that leaves is reported as left, healthy ranks
  are not reported;
* gloo ranks: a rank that raises before the collective, and one that never
  joins, make the others fail with an error within the process-group timeout
  (no hang), and the monitor tells the survivors which rank is gone;
* bad inputs are declined by the gating (misaligned size, dtype, layout,
  oversize) so the caller falls back to NCCL.
"""

import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from numa_allreduce_b200.parallel.health import PeerLost, PeerMonitor


def _store(world):
    from datetime import timedelta

    return dist.TCPStore("127.0.0.1", free_port(), world, True, timeout=timedelta(seconds=10),
                         wait_for_workers=False)


def test_monitor_reports_silent_rank():
    store = _store(3)
    mons = [PeerMonitor(store, r, 3, interval_s=0.05, timeout_s=0.5) for r in range(3)]
    mons[0].start()
    mons[1].start()  # rank 2 beat once at construction and then went silent
    try:
        # each monitor starts watching (a peer is judged from a rank's first look on)
        assert mons[0].dead_ranks() == [] and mons[1].dead_ranks() == []
        time.sleep(0.9)
        assert mons[0].dead_ranks() == [2]
        assert mons[1].dead_ranks() == [2]
        with pytest.raises(PeerLost) as e:
            mons[0].assert_healthy()
        assert e.value.dead == [2] and e.value.left == []
    finally:
        for m in mons:
            m.stop()


def test_monitor_reports_left_rank_and_never_joined():
    store = _store(3)
    a = PeerMonitor(store, 0, 3, interval_s=0.05, timeout_s=0.4).start()
    b = PeerMonitor(store, 1, 3, interval_s=0.05, timeout_s=0.4).start()
    try:
        b.leave()
        dead, left = a.status()
        assert left == [1]
        time.sleep(0.6)  # rank 2 never created its monitor
        dead, left = a.status()
        assert dead == [2] and left == [1]
    finally:
        a.stop()
        b.stop()


def test_monitor_rejects_bad_timing():
    with pytest.raises(ValueError):
        PeerMonitor(_store(1), 0, 1, interval_s=1.0, timeout_s=0.5)


def _worker_dead_peer(rank, world, port, mode, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    from numa_allreduce_b200.parallel.emulate import emulate_allreduce
    from numa_allreduce_b200.parallel.schedule import HierSchedule

    # the rendezvous may wait for slow interpreter start-up (a long bound);
    # only the collectives under test run on a group with a short timeout
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    group = dist.new_group(backend="gloo", timeout=timedelta(seconds=3))
    store = dist.distributed_c10d._get_default_store()
    mon = PeerMonitor(store, rank, world, interval_s=0.1, timeout_s=1.0).start()
    sched = HierSchedule.from_groups([[0, 1], [2, 3]] if world == 4 else [list(range(world))])
    x = torch.full((1024,), float(rank + 1))
    # one good step on every rank
    out = emulate_allreduce(x, sched, group)
    assert torch.all(out == sum(range(1, world + 1)))
    assert mon.status() == ([], [])  # checked every step
    dist.barrier(group=group)
    if rank == world - 1:
        if mode == "raise":
            mon.stop()
            os._exit(3)  # dies between steps, with nothing in flight
        mon.leave()  # "leave": clean exit announced through the store
        os._exit(0)
    # survivors: the next collective fails with an error, it does not hang
    t0 = time.monotonic()
    err = None
    try:
        emulate_allreduce(x, sched, group)
    except Exception as e:  # gloo reports the lost peer or the timeout
        err = type(e).__name__
    waited = time.monotonic() - t0
    time.sleep(1.5)  # the heartbeat timeout passes
    dead, left = mon.status()
    mon.stop()
    result_q.put((rank, err, waited, dead, left))
    result_q.close()
    result_q.join_thread()  # flush before the hard exit below
    os._exit(0)  # skip teardown collectives with a peer gone


@pytest.mark.parametrize("mode", ["raise", "leave"])
def test_gloo_rank_loss_fails_fast_and_is_named(mode):
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.monotonic() + 90
    while len(results) < world - 1 and time.monotonic() < deadline:
        try:
            results.append(q.get(timeout=5))
        except Exception:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(results) == world - 1, results
    for rank, err, waited, dead, left in results:
        assert err is not None, f"rank {rank}: the collective after the loss did not fail"
        assert waited < 20, f"rank {rank} waited {waited:.1f} s"
        if mode == "leave":
            assert left == [world - 1], (rank, dead, left)
        else:
            assert dead == [world - 1], (rank, dead, left)


class _GateOnly:
    """The gating of NumaAwareAllReduce, without devices (white-box)."""

    def __init__(self, max_size):
        from numa_allreduce_b200.parallel.comm import NumaAwareAllReduce
        from numa_allreduce_b200.parallel.select import AlgoSelector

        self.obj = object.__new__(NumaAwareAllReduce)
        self.obj.disabled = False
        self.obj.max_size = max_size
        self.obj.selector = AlgoSelector.load(8, has_nvls=False, has_groups=False)

    def ok(self, t):
        return self.obj.should_use_numa_ar(t)


def test_gating_declines_bad_inputs():
    g = _GateOnly(max_size=1 << 20)
    assert g.ok(torch.empty(1024, dtype=torch.bfloat16))
    assert not g.ok(torch.empty(1023, dtype=torch.bfloat16))        # not a multiple of 16 bytes
    assert not g.ok(torch.empty(1024, dtype=torch.int32))           # dtype
    assert g.ok(torch.empty(64, 64, dtype=torch.float32).t())       # dense in its storage: fine
    assert not g.ok(torch.empty(64, 64, dtype=torch.float32)[:, :32])  # a strided view: declined
    assert not g.ok(torch.empty(0, dtype=torch.float32))            # empty
    assert not g.ok(torch.empty(1 << 20, dtype=torch.float32))      # 4 MiB > max_size: NCCL
    g.obj.disabled = True
    assert not g.ok(torch.empty(1024, dtype=torch.bfloat16))
