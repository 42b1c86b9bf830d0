"""Reduce-scatter and all-gather collectives on CPU: the exact oracle and
the gloo executor of the same data movement (segment j to its owner j,
owner adds in rank order; own segment to every peer).

The GPU kernels are held to the same oracle in
tests/test_gpu_emulated_allreduce.py and tests/test_gpu_multiproc.py.
"""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from numa_allreduce_b200 import (HierSchedule, emulate_all_gather, emulate_reduce_scatter, reference_all_gather,
                                 reference_allreduce, reference_reduce_scatter)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ws", [2, 3, 8])
def test_reduce_scatter_oracle_is_the_allreduce_slice(ws, dtype):
    xs = [torch.randn(ws * 1000, generator=torch.Generator().manual_seed(r)).to(dtype) for r in range(ws)]
    full = reference_allreduce(xs, HierSchedule.oneshot(ws))
    outs = reference_reduce_scatter(xs)
    assert len(outs) == ws
    for r, o in enumerate(outs):
        assert o.dtype == dtype and o.numel() == 1000
        assert torch.equal(o, full[r * 1000:(r + 1) * 1000])


def test_reduce_scatter_oracle_rejects_ragged_inputs():
    with pytest.raises(ValueError):
        reference_reduce_scatter([torch.zeros(10), torch.zeros(10), torch.zeros(10)])  # 10 % 3 != 0
    with pytest.raises(ValueError):
        reference_reduce_scatter([torch.zeros(8), torch.zeros(6)])


def test_all_gather_oracle_order():
    xs = [torch.full((3, 2), float(r)) for r in range(4)]
    out = reference_all_gather(xs)
    assert out.shape == (24,)
    assert torch.equal(out.view(4, 6), torch.arange(4.0).repeat_interleave(6).view(4, 6))


def _worker(rank, ws, port, dtype_name, seg, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        dtype = getattr(torch, dtype_name)
        torch.manual_seed(rank)
        x = torch.randn(ws * seg, dtype=torch.float32).to(dtype)
        everyone = [torch.empty(ws * seg) for _ in range(ws)]
        dist.all_gather(everyone, x.float())  # fp32 round trip is exact
        inputs = [e.to(dtype) for e in everyone]
        rs = emulate_reduce_scatter(x, group=None)
        rs_exact = torch.equal(rs, reference_reduce_scatter(inputs)[rank])
        expected = x.float().clone()
        dist.all_reduce(expected)
        rs_err = (rs.float() - expected[rank * seg:(rank + 1) * seg]).abs().max().item()
        mine = x[:seg].contiguous()
        ag = emulate_all_gather(mine, group=None)
        ag_exact = torch.equal(ag, reference_all_gather([i[:seg] for i in inputs]))
        result_q.put((rank, rs_exact, rs_err, ag_exact, rs.numel(), ag.numel()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws,dtype_name", [(2, "float32"), (4, "bfloat16"), (3, "float16")])
def test_gloo_collectives_match_oracle(ws, dtype_name):
    seg = 1031
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker, args=(ws, free_port(), dtype_name, seg, q), nprocs=ws, join=True)
    res = [q.get(timeout=60) for _ in range(ws)]
    tol = 1e-5 if dtype_name == "float32" else 0.05
    for rank, rs_exact, rs_err, ag_exact, n_rs, n_ag in res:
        assert rs_exact, f"rank {rank}: reduce-scatter not bit-exact"
        assert rs_err <= tol * ws, f"rank {rank}: reduce-scatter error {rs_err}"
        assert ag_exact, f"rank {rank}: all-gather differs"
        assert n_rs == seg and n_ag == ws * seg


def _bare(ws):
    """A NumaAwareAllReduce without a device: enough for the argument checks."""
    from numa_allreduce_b200 import NumaAwareAllReduce

    ar = object.__new__(NumaAwareAllReduce)
    ar.disabled = False
    ar.world_size = ws
    return ar


def test_collective_argument_checks():
    ar = _bare(4)
    seg = torch.zeros(8, dtype=torch.bfloat16)      # 16 bytes: the smallest valid segment
    big = torch.zeros(32, dtype=torch.bfloat16)
    ar._check_collective(seg, big)                   # fine
    with pytest.raises(ValueError, match="world_size"):
        ar._check_collective(seg, torch.zeros(24, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="16 bytes"):
        ar._check_collective(torch.zeros(4, dtype=torch.bfloat16), torch.zeros(16, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="dtype"):
        ar._check_collective(seg, big.float())
    with pytest.raises(ValueError, match="dtype"):
        ar._check_collective(seg.to(torch.int16), big.to(torch.int16))
    with pytest.raises(ValueError, match="contiguous"):
        ar._check_collective(torch.zeros(16, dtype=torch.bfloat16)[::2], big)
    ar.disabled = True
    with pytest.raises(RuntimeError, match="disabled"):
        ar._check_collective(seg, big)


def test_custom_collectives_hand_large_or_odd_messages_to_nccl(monkeypatch):
    """custom_reduce_scatter / custom_all_gather return None ("use NCCL") above
    the segment cap and for inputs the kernel cannot take; otherwise they run
    the collective (stubbed here: no GPU)."""
    from numa_allreduce_b200.utils.env import read_env

    ar = _bare(4)
    ar.env = read_env()
    assert ar.env.collective_max == 1 << 20
    calls = []
    monkeypatch.setattr(type(ar), "reduce_scatter", lambda self, x, out=None: calls.append(("rs", x.numel())) or x)
    monkeypatch.setattr(type(ar), "all_gather", lambda self, x, out=None: calls.append(("ag", x.numel())) or x)
    bf = torch.bfloat16
    assert ar.custom_reduce_scatter(torch.zeros(4 * 8, dtype=bf)) is not None           # 16-byte segments
    assert ar.custom_reduce_scatter(torch.zeros(4 * (1 << 19), dtype=bf)) is not None   # 1 MiB segments
    assert ar.custom_reduce_scatter(torch.zeros(4 * (1 << 19) + 32, dtype=bf)) is None  # above the cap
    assert ar.custom_reduce_scatter(torch.zeros(30, dtype=bf)) is None                  # not 4 segments
    assert ar.custom_reduce_scatter(torch.zeros(4 * 4, dtype=bf)) is None               # 8-byte segments
    assert ar.custom_reduce_scatter(torch.zeros(64, dtype=torch.int32)) is None         # dtype
    assert ar.custom_reduce_scatter(torch.zeros(128, dtype=bf)[::2]) is None            # not contiguous
    assert ar.custom_all_gather(torch.zeros(1 << 19, dtype=bf)) is not None
    assert ar.custom_all_gather(torch.zeros((1 << 19) + 8, dtype=bf)) is None
    assert calls == [("rs", 32), ("rs", 4 << 19), ("ag", 1 << 19)]
    monkeypatch.setenv("NAB_COLLECTIVE_MAX", str(64 << 20))
    ar.env = read_env()
    assert ar.custom_reduce_scatter(torch.zeros(4 * (1 << 20), dtype=bf)) is not None
    ar.disabled = True
    assert ar.custom_all_gather(torch.zeros(8, dtype=bf)) is None
