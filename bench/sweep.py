#!/usr/bin/env python3
"""Allreduce sweep: p50 latency and bus bandwidth per protocol, dtype and size.

Contiguous 1-D tensors of 4 KiB .. 256 MiB (powers
of two), N(0,1) with seed = rank, every protocol of this library plus NCCL and
the reference's custom allreduce (``--ref``), 200 timed iterations after 20
warm-up. Launch with torch.distributed.run, one process per GPU::

    python -m torch.distributed.run --nproc-per-node 8 bench/sweep.py --dtypes bf16 --ref

Modes: ``eager`` times back-to-back launches with CUDA events around every call
(p50 over calls, max over ranks); ``graph`` captures ``--graph-calls`` calls of
this library's kernels in one CUDA graph and reports replay time per call, i.e.
device time without host launch overhead. ``--write-table`` turns the eager
results into the selector's JSON tuning table.
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
from numa_allreduce_b200.parallel.select import build_table  # noqa: E402
from numa_allreduce_b200.utils.timing import busbw_gbs  # noqa: E402

DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--sizes", default=",".join(str(4096 << i) for i in range(17)))
    p.add_argument("--dtypes", default="bf16")
    p.add_argument("--algos", default="auto", help="comma list, 'all' or 'auto' (selector)")
    p.add_argument("--iters", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--mode", choices=["eager", "graph", "both"], default="both")
    p.add_argument("--graph-calls", type=int, default=20)
    p.add_argument("--nccl", action="store_true", default=True)
    p.add_argument("--no-nccl", dest="nccl", action="store_false")
    p.add_argument("--ref", action="store_true", help="include the reference's custom allreduce")
    p.add_argument("--out", default=None)
    p.add_argument("--write-table", default=None)
    p.add_argument("--max-oneshot", type=int, default=1 << 20)
    p.add_argument("--hier-groups", default=None, help="e.g. 0,1,2,3|4,5,6,7")
    p.add_argument("--pipe-configs", default=None,
                   help="extra pipelined two-shot configurations to time, e.g. 148x256,128x512 (CTAs x tile KiB)")
    p.add_argument("--oneshot-configs", default=None,
                   help="extra one-shot launch shapes to time up to 1 MiB, e.g. 256x64,512x32 (packs per CTA x max CTAs)")
    p.add_argument("--hybrid-configs", default=None,
                   help="hybrid splits to time, e.g. 400x64x80,300x56x88 (P2P per mille x P2P CTAs x NVLS CTAs); "
                        "--write-table keeps the one with the best bus bandwidth summed over sizes >= 16 MiB")
    p.add_argument("--nvlink", action="store_true",
                   help="read the NVLink traffic counters around each eager timing (bytes per call per direction)")
    p.add_argument("--merge", action="store_true",
                   help="--write-table replaces only the entries it measured in an existing table")
    return p.parse_args()


def pick_hybrid(rows):
    """Best hybrid split of a sweep: highest bus bandwidth summed over the
    sizes of at least 16 MiB. Returns (split, rows relabelled "hybrid")."""
    score = {}
    for r in rows:
        if r["algo"].startswith("hybrid:") and r["bytes"] >= (16 << 20):
            score[r["algo"]] = score.get(r["algo"], 0.0) + r["busbw_gbs"]
    if not score:
        return None, [r for r in rows if not r["algo"].startswith("hybrid:")]
    best = max(score, key=score.get)
    split = tuple(int(v) for v in best.split(":")[1].split("x"))
    out = []
    for r in rows:
        if r["algo"].startswith("hybrid:"):
            if r["algo"] == best:
                out.append(dict(r, algo="hybrid"))
        elif r["algo"] != "hybrid":
            out.append(r)
    return split, out


def merge_tables(old: dict, new: dict) -> dict:
    """``new``'s entries replace ``old``'s of the same (world size, dtype,
    nvls); a hybrid split in ``new`` replaces the one of its world size."""
    keys = {(e["world_size"], e["dtype"], e["nvls"]) for e in new.get("entries", [])}
    entries = [e for e in old.get("entries", []) if (e["world_size"], e["dtype"], e["nvls"]) not in keys]
    entries += new.get("entries", [])
    entries.sort(key=lambda e: (e["world_size"], e["dtype"], e["nvls"]))
    out = {"version": 1, "entries": entries}
    hyb = dict(old.get("hybrid", {}))
    hyb.update(new.get("hybrid", {}))
    if hyb:
        out["hybrid"] = hyb
    return out


def max_over_ranks(vals):
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def time_eager(fn, iters, warmup, counters=None):
    """p50 device time per call (us); with ``counters`` also the NVLink
    bytes per call per direction read around the timed calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    before = counters.read() if counters else None
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    link = None
    if counters:
        from numa_allreduce_b200.utils.nvlink import delta

        link = delta(before, counters.read(), iters)
    return statistics.median(a.elapsed_time(b) * 1e3 for a, b in ev), link


def time_graph(fn, calls, reps, warmup):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    for _ in range(max(1, warmup // calls)):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (reps * calls)
    del g
    return us


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    groups = None
    if args.hier_groups:
        from numa_allreduce_b200.utils.env import parse_groups

        groups = parse_groups(args.hier_groups)
    ar = NumaAwareAllReduce(dist.group.WORLD, device=local, hier_groups=groups, oneshot_max=args.max_oneshot)
    ref = None
    if args.ref:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        try:
            from ref_arm import load_reference_class

            gloo = dist.new_group(backend="gloo")
            ref = load_reference_class()(group=gloo, device=local)
            if ref.disabled:
                ref = None
        except Exception as e:
            if rank == 0:
                print(f"reference unavailable: {e}", flush=True)
            ref = None
    extra = []
    if args.pipe_configs:
        for spec in args.pipe_configs.split(","):
            ctas, tile_kib = (int(v) for v in spec.split("x"))
            extra.append((f"pipe_{ctas}x{tile_kib}",
                          NumaAwareAllReduce(dist.group.WORLD, device=local, use_nvls=False, pipe_ctas=ctas,
                                             pipe_tile=tile_kib << 10)))
    counters = None
    if args.nvlink and rank == 0:
        try:
            from numa_allreduce_b200.utils.nvlink import NvlinkCounters
            from numa_allreduce_b200.utils.timing import pci_bus_id

            counters = NvlinkCounters(pci_bus_id(local))
            counters.read()
            print(f"NVLink counters: links {counters.links}, diagnostics {counters.diag}", flush=True)
        except Exception as e:  # counters are optional
            print(f"NVLink counters unavailable: {e}", flush=True)
    oneshot_extra = []
    if args.oneshot_configs:
        for spec in args.oneshot_configs.split(","):
            grain, ctas = (int(v) for v in spec.split("x"))
            oneshot_extra.append((f"oneshot_{grain}x{ctas}",
                                  NumaAwareAllReduce(dist.group.WORLD, device=local, use_nvls=False,
                                                     oneshot_grain=grain, oneshot_ctas=ctas)))
    sizes = [int(v) for v in args.sizes.split(",")]
    if args.algos == "all":
        algos = ["oneshot", "twoshot", "twoshot_pipe"] + (
            ["nvls_oneshot", "nvls_twoshot"] + ([] if args.hybrid_configs else ["hybrid"]) if ar.has_nvls else []) + \
                (["hier"] if ar.hier_groups else [])
    elif args.algos == "auto":
        algos = ["auto"]
    else:
        algos = args.algos.split(",")
    rows = []
    for dname in args.dtypes.split(","):
        dtype = DT[dname]
        esize = torch.tensor([], dtype=dtype).element_size()
        for size in sizes:
            n = size // esize
            g = torch.Generator(device="cuda").manual_seed(rank)
            x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32).to(dtype)
            out = torch.empty_like(x)
            expect = x.float().clone()  # for fp32, x.float() is x itself
            dist.all_reduce(expect)
            cands = []
            for algo in algos:
                name = ar.algo_for(size, dtype) if algo == "auto" else algo
                if name in ("oneshot", "nvls_oneshot") and size > args.max_oneshot:
                    continue
                if name == "nccl":
                    continue
                cands.append((algo if algo != "auto" else f"auto:{name}",
                              (lambda nm=name: ar.all_reduce(x, out=out, algo=nm)), True))
            for label, comm in extra:
                cands.append((label, (lambda c=comm: c.all_reduce(x, out=out, algo="twoshot_pipe")), True))
            if size <= args.max_oneshot:
                for label, comm in oneshot_extra:
                    cands.append((label, (lambda c=comm: c.all_reduce(x, out=out, algo="oneshot")), True))
            if args.hybrid_configs and ar.has_nvls:
                for spec in args.hybrid_configs.split(","):
                    split = tuple(int(v) for v in spec.split("x"))

                    def run_hybrid(split=split):
                        ar.set_hybrid(*split)
                        return ar.all_reduce(x, out=out, algo="hybrid")
                    cands.append((f"hybrid:{spec}", run_hybrid, True))
            if args.nccl:
                y = x.clone()
                cands.append(("nccl", lambda: dist.all_reduce(y), False))
            if ref is not None and ref.should_use_numa_ar(x):
                cands.append(("ref_custom_ar", lambda: ref.custom_all_reduce(x), False))
            for label, fn, ours in cands:
                ok = True
                if ours:
                    fn()
                    torch.cuda.synchronize()
                    ar.check()
                    tol = 1e-5 * world if dtype == torch.float32 else 2e-2 * world
                    ok = bool(torch.allclose(out.float(), expect, rtol=1e-2, atol=tol))
                flag = torch.tensor([1 if ok else 0], device="cuda")
                dist.all_reduce(flag, op=dist.ReduceOp.MIN)
                modes = ["eager"] if not ours or args.mode == "eager" else (
                    ["graph"] if args.mode == "graph" else ["eager", "graph"])
                if not ours and args.mode == "graph":
                    modes = []
                for mode in modes:
                    link = None
                    if mode == "eager":
                        us, link = time_eager(fn, args.iters, args.warmup, counters)
                    else:
                        reps = max(1, args.iters // args.graph_calls)
                        us = time_graph(fn, args.graph_calls, reps, args.warmup)
                    us = max_over_ranks([us])[0]
                    row = {"world_size": world, "dtype": NAMES[dtype], "bytes": size, "algo": label,
                           "mode": mode, "p50_us": round(us, 2), "busbw_gbs": round(busbw_gbs(size, us / 1e6, world), 1),
                           "nvls": ar.has_nvls, "correct": bool(flag.item())}
                    if link is not None:
                        row["nvlink_per_call"] = {k: None if v is None else [round(v[0]), round(v[1])]
                                                  for k, v in link.items()}
                    rows.append(row)
                    if rank == 0:
                        extra_txt = f" nvlink/call {row['nvlink_per_call']}" if "nvlink_per_call" in row else ""
                        print(f"{NAMES[dtype]:>8} {size:>11} {label:>22} {mode:>5} {us:10.2f} us "
                              f"{row['busbw_gbs']:8.1f} GB/s {'ok' if row['correct'] else 'WRONG'}{extra_txt}",
                              flush=True)
    if rank == 0:
        if args.out:
            with open(args.out, "w") as f:
                json.dump({"world_size": world, "nvls": ar.has_nvls, "rows": rows}, f, indent=1)
        if args.write_table:
            tab_rows = [dict(r, algo=r["algo"].split(":")[-1] if r["algo"].startswith("auto:") else r["algo"])
                        for r in rows
                        if r["mode"] == "eager" and r["correct"]
                        and not r["algo"].startswith(("ref", "pipe_", "oneshot_"))]
            split, tab_rows = pick_hybrid(tab_rows)
            table = build_table(tab_rows, hybrid={world: split} if split else None)
            if args.merge and os.path.exists(args.write_table):
                table = merge_tables(json.load(open(args.write_table)), table)
            with open(args.write_table, "w") as f:
                json.dump(table, f, indent=1)
    torch.cuda.synchronize()
    ar.close()
    for _, comm in extra + oneshot_extra:
        comm.close()
    if ref is not None:
        ref.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
