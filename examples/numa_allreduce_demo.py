#!/usr/bin/env python3
"""Demo of NumaAwareAllReduce: topology, a correctness check and a benchmark.

The same three parts as the reference's demo (examples/numa_allreduce_demo.py:
topology print, correctness against NCCL on fp32 tensors of 4 and 64 MB,
benchmark at 64/256/1024 MB), with device-side timing: every number is CUDA
events on the launching stream, after warm-up, maximum over ranks.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        examples/numa_allreduce_demo.py [--sizes-mb 64,256,1024] [--dtype bf16]
"""

from __future__ import annotations

import argparse
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from numa_allreduce_b200 import NumaAwareAllReduce, NumaTopology  # noqa: E402
from numa_allreduce_b200.utils.timing import busbw_gbs  # noqa: E402

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--check-mb", default="4,64", help="sizes (MB) of the correctness check")
    p.add_argument("--sizes-mb", default="64,256,1024", help="sizes (MB) of the benchmark")
    p.add_argument("--dtype", default="bf16", choices=sorted(DTYPES))
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    return p.parse_args()


def max_over_ranks(x: float) -> float:
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def timed(fn, iters: int, warmup: int) -> float:
    """Median per-call device time in microseconds, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    us = sorted(a.elapsed_time(b) * 1e3 for a, b in times)[len(times) // 2]
    return max_over_ranks(us)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ar = NumaAwareAllReduce(dist.group.WORLD, device=local)
    if rank == 0:
        print("== topology ==")
        print(NumaTopology.detect().get_summary())
        print(f"custom allreduce: {'disabled' if ar.disabled else 'enabled'}, world size {world}, "
              f"NVLS {'on' if ar.has_nvls else 'off'}, groups {ar.get_numa_groups()}")

    # correctness against NCCL, fp32 (as the reference checks it)
    ok = True
    for mb in [float(s) for s in args.check_mb.split(",")]:
        n = int(mb * (1 << 20)) // 4
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32)
        ref = x.clone()
        dist.all_reduce(ref)
        out = ar.custom_all_reduce(x)
        if out is None:
            res = "NCCL fallback (custom path declined the message)"
        else:
            torch.cuda.synchronize()
            err = (out - ref).abs().max().item()
            good = err <= 1e-3
            ok &= good
            res = f"max |custom - NCCL| = {err:.2e} {'OK' if good else 'MISMATCH'}"
        if rank == 0:
            print(f"check fp32 {mb:g} MB: {res}")

    # benchmark
    dt = DTYPES[args.dtype]
    if rank == 0:
        print(f"== benchmark ({args.dtype}, median of {args.iters}, max over {world} ranks) ==")
        print(f"{'size':>10} {'algo':>14} {'custom us':>10} {'busbw':>8} {'NCCL us':>10} {'busbw':>8} {'speedup':>8}")
    for mb in [float(s) for s in args.sizes_mb.split(",")]:
        n = int(mb * (1 << 20)) // torch.tensor([], dtype=dt).element_size()
        x = torch.randn(n, device="cuda").to(dt)
        y = x.clone()
        nbytes = n * x.element_size()
        algo = ar.algo_for(nbytes, dt) if not ar.disabled else "nccl"
        t_nccl = timed(lambda: dist.all_reduce(y), args.iters, args.warmup)
        if algo != "nccl":
            out = torch.empty_like(x)
            t_ours = timed(lambda: ar.all_reduce(x, out), args.iters, args.warmup)
        else:
            t_ours = t_nccl
        if rank == 0:
            print(f"{mb:>8g}MB {algo:>14} {t_ours:>10.1f} {busbw_gbs(nbytes, t_ours * 1e-6, world):>8.1f} "
                  f"{t_nccl:>10.1f} {busbw_gbs(nbytes, t_nccl * 1e-6, world):>8.1f} {t_nccl / t_ours:>8.2f}")
        del x, y
    ar.check()
    torch.cuda.synchronize()
    ar.close()
    dist.destroy_process_group()
    if not ok:
        sys.exit(1)


if __name__ == "__main__":
    main()
