#!/usr/bin/env python3
"""Reduce-scatter and all-gather: this library's segment collectives against
NCCL (``reduce_scatter_tensor`` / ``all_gather_into_tensor``).

Sizes are the bytes of ONE rank's segment (the reduce-scatter input and the
all-gather output are world_size segments). p50 device time per call over
``--iters`` eager calls (CUDA events around each call, max over ranks), and
bus bandwidth S (ws - 1) / ws / t with S = one segment's bytes times world
size, the convention of nccl-tests. Every result is checked against NCCL first.
Launch with torch.distributed.run, one process per GPU::

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 bench/collectives.py
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from numa_allreduce_b200 import NumaAwareAllReduce  # noqa: E402


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--sizes", default=",".join(str(4096 << i) for i in range(0, 15, 2)))
    p.add_argument("--iters", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--out", default=None)
    return p.parse_args()


def time_eager(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) * 1e3 for a, b in ev)


def max_over_ranks(vals):
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def main():
    a = parse()
    rank = int(os.environ.get("RANK", 0))
    ws = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ar = NumaAwareAllReduce(dist.group.WORLD, device=local)
    rows = []
    try:
        for seg_bytes in [int(s) for s in a.sizes.split(",")]:
            seg = seg_bytes // 2
            torch.manual_seed(rank)
            x = torch.randn(ws * seg, dtype=torch.bfloat16, device="cuda")
            rs_out = torch.empty(seg, dtype=torch.bfloat16, device="cuda")
            rs_ref = torch.empty_like(rs_out)
            mine = x[:seg].contiguous()
            ag_out = torch.empty(ws * seg, dtype=torch.bfloat16, device="cuda")
            ag_ref = torch.empty_like(ag_out)
            ar.reduce_scatter(x, rs_out)
            dist.reduce_scatter_tensor(rs_ref, x)
            ar.all_gather(mine, ag_out)
            dist.all_gather_into_tensor(ag_ref, mine)
            torch.cuda.synchronize()
            ar.check()
            ok = bool(torch.allclose(rs_out.float(), rs_ref.float(), rtol=1e-2, atol=1e-2 * ws)
                      and torch.equal(ag_out, ag_ref))
            t = [time_eager(lambda: ar.reduce_scatter(x, rs_out), a.iters, a.warmup),
                 time_eager(lambda: dist.reduce_scatter_tensor(rs_ref, x), a.iters, a.warmup),
                 time_eager(lambda: ar.all_gather(mine, ag_out), a.iters, a.warmup),
                 time_eager(lambda: dist.all_gather_into_tensor(ag_ref, mine), a.iters, a.warmup)]
            t = max_over_ranks(t)
            ok_all = torch.tensor([1 if ok else 0], device="cuda")
            dist.all_reduce(ok_all, op=dist.ReduceOp.MIN)
            total = seg_bytes * ws

            def bus(us):
                return round(total * (ws - 1) / ws / (us * 1e-6) / 1e9, 1)

            row = {"world_size": ws, "segment_bytes": seg_bytes, "correct": bool(ok_all.item()),
                   "rs_us": round(t[0], 2), "rs_nccl_us": round(t[1], 2), "ag_us": round(t[2], 2),
                   "ag_nccl_us": round(t[3], 2), "rs_busbw_gbs": bus(t[0]), "rs_nccl_busbw_gbs": bus(t[1]),
                   "ag_busbw_gbs": bus(t[2]), "ag_nccl_busbw_gbs": bus(t[3])}
            rows.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
    finally:
        torch.cuda.synchronize()
        ar.close()
    if rank == 0 and a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
