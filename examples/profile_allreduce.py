#!/usr/bin/env python3
"""Profiling front end for the allreduce (the reference's
examples/profile_nsys_ncu.py: benchmark, NVTX-annotated and ncu modes).

Modes:

  benchmark  device-timed median per call of this library and of NCCL for one
             message size; algbw = S/t and busbw = S/t * 2(n-1)/n (the
             reference printed 2S/t, which is neither), max over ranks.
  nvtx       the same loops inside NVTX ranges ``nab/<algo>`` / ``nccl`` with
             one sub-range per iteration, for a timeline profiler.
  ncu        a short fixed number of this library's calls and nothing else, to
             run under ``ncu`` on ONE process (``--single`` emulates the
             ranks inside one process on one GPU, so no multi-rank job is
             wrapped in the profiler). Always give ncu ``--clock-control none``:

      python examples/profile_allreduce.py --mode ncu --single --ranks 8 --size-mb 16 > plain.log && \\
      ncu --set full --clock-control none -k regex:k_twoshot -c 1 -o prof \\
          python examples/profile_allreduce.py --mode ncu --single --ranks 8 --size-mb 16

Multi-rank modes are launched with torch.distributed.run, one process per GPU.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from numa_allreduce_b200.utils.timing import algbw_gbs, busbw_gbs  # noqa: E402

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--mode", default="benchmark", choices=["benchmark", "nvtx", "ncu"])
    p.add_argument("--size-mb", type=float, default=64.0)
    p.add_argument("--dtype", default="bf16", choices=sorted(DTYPES))
    p.add_argument("--algo", default=None, help="force a protocol (default: the selector's choice)")
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--single", action="store_true", help="emulate --ranks ranks on one GPU (ncu mode)")
    p.add_argument("--ranks", type=int, default=8)
    p.add_argument("--op", default="allreduce", choices=["allreduce", "fused", "reduce_scatter", "all_gather"],
                   help="--single: the allreduce, the fused allreduce + residual + RMSNorm, or a segment "
                        "collective (--size-mb is then one rank's segment)")
    p.add_argument("--tokens", type=int, default=16, help="--op fused: rows T of the [T, hidden] message")
    p.add_argument("--hidden", type=int, default=8192, help="--op fused: hidden size H")
    p.add_argument("--groups", default=None, help="--single with --algo hier: e.g. 0,1,2,3|4,5,6,7")
    return p.parse_args()


def single_gpu(args):
    """ncu-friendly: one process, one GPU, the ranks emulated by one launch.
    Device time per call (CUDA events, median) is printed with the call."""
    from numa_allreduce_b200.ops.allreduce import EmulatedGroup
    from numa_allreduce_b200.utils.env import parse_groups

    dt = DTYPES[args.dtype]
    algo = args.algo or ("twoshot" if args.op == "allreduce" else "auto")
    groups = parse_groups(args.groups) if args.groups else None
    iters = 3 if args.mode == "ncu" else args.iters
    # the emulation runs at most 148 / ranks CTAs per rank: size the rings for that
    with EmulatedGroup(args.ranks, groups=groups, pipe_ctas=max(1, 148 // args.ranks),
                       fused_bytes=max(512 << 10, args.tokens * args.hidden * 2)) as grp:
        if args.op == "allreduce":
            n = int(args.size_mb * (1 << 20)) // torch.tensor([], dtype=dt).element_size()
            ins = [torch.randn(n, device="cuda").to(dt) for _ in range(args.ranks)]
            outs = [torch.empty_like(x) for x in ins]
            nbytes = n * ins[0].element_size()

            def call():
                grp.all_reduce(ins, algo=algo, outs=outs)
        elif args.op in ("reduce_scatter", "all_gather"):
            seg = int(args.size_mb * (1 << 20)) // torch.tensor([], dtype=dt).element_size()
            rs = args.op == "reduce_scatter"
            ins = [torch.randn(seg * (args.ranks if rs else 1), device="cuda").to(dt) for _ in range(args.ranks)]
            outs = [torch.empty(seg * (1 if rs else args.ranks), device="cuda", dtype=dt) for _ in range(args.ranks)]
            nbytes = seg * ins[0].element_size()
            algo = args.op

            def call():
                getattr(grp, args.op)(ins, outs=outs)
        else:
            T, H = args.tokens, args.hidden
            ins = [torch.randn(T, H, device="cuda").to(torch.bfloat16) for _ in range(args.ranks)]
            res = [torch.randn(T, H, device="cuda").to(torch.bfloat16) for _ in range(args.ranks)]
            wts = [torch.ones(H, device="cuda", dtype=torch.bfloat16) for _ in range(args.ranks)]
            outs = [torch.empty_like(x) for x in ins]
            nbytes = T * H * 2

            def call():
                grp.fused_ar_rmsnorm(ins, res, wts, eps=1e-5, algo=algo, outs=outs)
        call()  # first call outside the timing
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            call()
            b.record()
            times.append((a, b))
        torch.cuda.synchronize()
        if any(grp.error_codes()):
            raise RuntimeError(f"emulated {args.op} reported errors: {grp.error_states()}")
        us = sorted(a.elapsed_time(b) * 1e3 for a, b in times)[len(times) // 2]
    print(json.dumps({"mode": args.mode, "single": True, "op": args.op, "ranks": args.ranks, "algo": algo,
                      "bytes_per_rank": nbytes, "us_per_call": round(us, 2)}))


def multi_rank(args):
    import torch.distributed as dist

    from numa_allreduce_b200 import NumaAwareAllReduce

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ar = NumaAwareAllReduce(dist.group.WORLD, device=local)
    dt = DTYPES[args.dtype]
    n = int(args.size_mb * (1 << 20)) // torch.tensor([], dtype=dt).element_size()
    x = torch.randn(n, device="cuda").to(dt)
    out = torch.empty_like(x)
    y = x.clone()
    nbytes = n * x.element_size()
    algo = args.algo or ar.algo_for(nbytes, dt)
    nvtx = args.mode == "nvtx"

    def loop(name, fn, iters):
        events = []
        if nvtx:
            torch.cuda.nvtx.range_push(name)
        for i in range(iters):
            if nvtx:
                torch.cuda.nvtx.range_push(f"{name}/iter{i}")
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            events.append((a, b))
            if nvtx:
                torch.cuda.nvtx.range_pop()
        if nvtx:
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        us = sorted(a.elapsed_time(b) * 1e3 for a, b in events)[len(events) // 2]
        t = torch.tensor([us], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    iters = 3 if args.mode == "ncu" else args.iters
    res = {"mode": args.mode, "world_size": world, "bytes": nbytes, "dtype": args.dtype, "algo": algo}
    if algo != "nccl" and not ar.disabled:
        loop("nab/warmup", lambda: ar.all_reduce(x, out, algo=algo), args.warmup)
        t = loop(f"nab/{algo}", lambda: ar.all_reduce(x, out, algo=algo), iters)
        res.update(custom_us=round(t, 2), custom_algbw=round(algbw_gbs(nbytes, t * 1e-6), 1),
                   custom_busbw=round(busbw_gbs(nbytes, t * 1e-6, world), 1))
    if args.mode != "ncu":
        loop("nccl/warmup", lambda: dist.all_reduce(y), args.warmup)
        t = loop("nccl", lambda: dist.all_reduce(y), iters)
        res.update(nccl_us=round(t, 2), nccl_algbw=round(algbw_gbs(nbytes, t * 1e-6), 1),
                   nccl_busbw=round(busbw_gbs(nbytes, t * 1e-6, world), 1))
    ar.check()
    if rank == 0:
        print(json.dumps(res), flush=True)
    torch.cuda.synchronize()
    ar.close()
    dist.destroy_process_group()


def main():
    args = parse()
    if args.mode == "ncu" and not args.single:
        sys.exit("--mode ncu runs under a profiler: use --single (one process, ranks emulated on one GPU)")
    if args.single:
        single_gpu(args)
    else:
        multi_rank(args)


if __name__ == "__main__":
    main()
