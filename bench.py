#!/usr/bin/env python3
"""Headline benchmark: bf16 allreduce across a sweep of message sizes.

Metric: "bf16 allreduce p50 us & bus GB/s vs msg size at
2/4/8 B200 vs ref & NCCL". One *step* is one out-of-place bf16 allreduce of
each of 17 contiguous 1-D messages of 4 KiB .. 256 MiB (powers of two) per
rank, N(0,1) data with seed = rank. ``value`` is the whole-job aggregate
algorithm bandwidth: n_gpus x (bytes per rank per step) / (device time per
step), in GB/s; the per-size p50 latency and bus bandwidth are in ``sweep``.
Device times are CUDA events on the launching stream, maximum over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run. The
reference arm runs the unmodified reference NumaAwareAllReduce (installed in
baseline/_ref) through its public ``custom_all_reduce``; where it returns
``None`` (messages above vLLM's sm_100 cap, or world size 1) the caller's
NCCL ``all_reduce`` runs, as the reference's own tests do.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import statistics
import sys
import time
import traceback
from datetime import timedelta

import torch
import torch.distributed as dist

METRIC = "bf16 allreduce p50 µs & bus GB/s vs msg size at 2/4/8 B200 vs ref & NCCL"
SIZES = [4096 << i for i in range(17)]  # 4 KiB .. 256 MiB


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--sizes", type=str, default=None, help="comma-separated bytes per rank")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="skip the per-size CUDA-graph replay timing")
    return p.parse_args()


def setup(n: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if "MASTER_PORT" not in os.environ:
        os.environ["MASTER_PORT"] = str(_free_port())
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    return rank, world, local


class OursArm:
    name = "ours"

    def __init__(self, local: int, sizes):
        from numa_allreduce_b200 import NumaAwareAllReduce

        self.ar = NumaAwareAllReduce(dist.group.WORLD, device=local)
        if self.ar.disabled:
            raise RuntimeError("custom allreduce is disabled")
        self.algos = {s: self.ar.algo_for(s, torch.bfloat16) for s in sizes}

    def step_one(self, x, out, s):
        if self.algos[s] == "nccl":
            # the selector hands this size to NCCL: the caller's in-place
            # all_reduce, exactly as the reference arm (and its tests) do
            dist.all_reduce(x)
            return x
        return self.ar.all_reduce(x, out=out)

    def launches(self) -> int:
        return self.ar.launches

    def capture(self, x, out, s, calls):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(calls):
                self.step_one(x, out, s)
        return g

    def close(self):
        self.ar.close()


class ReferenceArm:
    name = "reference"

    def __init__(self, local: int, sizes):
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline"))
        from ref_arm import load_reference_class

        cls = load_reference_class()
        self.gloo = dist.new_group(backend="gloo")
        self.ar = cls(group=self.gloo, device=local)
        self.algos = {}
        for s in sizes:
            probe = torch.empty(s // 2, dtype=torch.bfloat16, device="cuda")
            self.algos[s] = "vllm_custom_ar" if (not self.ar.disabled and self.ar.should_use_numa_ar(probe)) \
                else "nccl"

    def step_one(self, x, out, s):
        r = self.ar.custom_all_reduce(x)
        if r is None:
            dist.all_reduce(x)
            return x
        return r

    def launches(self):
        return None

    def capture(self, x, out, s, calls):
        """The reference's own capture flow (src/numa_all_reduce.py:362-413):
        a warm-up call inside ``capture()``, then the graph; leaving the
        context registers the captured buffers on every rank."""
        g = torch.cuda.CUDAGraph()
        with self.ar.capture():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.step_one(x, out, s)
            torch.cuda.current_stream().wait_stream(side)
            with torch.cuda.graph(g):
                for _ in range(calls):
                    self.step_one(x, out, s)
        return g

    def close(self):
        if not self.ar.disabled:
            self.ar.close()


def _max_over_ranks(values: list[float]) -> list[float]:
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _sum_over_ranks(v: int) -> int:
    t = torch.tensor([v], dtype=torch.int64, device="cuda")
    dist.all_reduce(t)
    return int(t.item())


def timed_sweep(arm, xs, outs, sizes, steps, warmup, rank, bus_ids):
    from numa_allreduce_b200.utils.timing import ClockSampler

    for _ in range(warmup):
        for s in sizes:
            arm.step_one(xs[s], outs[s], s)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev = {s: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)] for s in sizes}
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(bus_ids).start() if rank == 0 and os.environ.get("NAB_BENCH_NO_CLOCKS") != "1" else None
    dist.barrier()
    torch.cuda.synchronize()
    l0 = arm.launches()
    t_host0 = time.time()
    start.record()
    for k in range(steps):
        for s in sizes:
            a, b = ev[s][k]
            a.record()
            arm.step_one(xs[s], outs[s], s)
            b.record()
    end.record()
    torch.cuda.synchronize()
    t_host1 = time.time()
    l1 = arm.launches()
    dist.barrier()
    clocks = sampler.stop(t_host0, t_host1) if sampler else None
    total_ms = start.elapsed_time(end)
    p50 = [statistics.median(a.elapsed_time(b) * 1e3 for a, b in ev[s]) for s in sizes]
    maxed = _max_over_ranks([total_ms] + p50)
    launches = None if l0 is None else _sum_over_ranks(l1 - l0)
    return maxed[0], maxed[1:], clocks, launches


def timed_graph(arm, xs, outs, sizes, calls=10, reps=5):
    """Per-size device time per call with the calls replayed from a CUDA graph
    (no host launch gap between them): ``calls`` calls captured once, the
    graph replayed ``reps`` times, max over ranks. Every rank captures the
    same sizes; a size whose capture failed on any rank reports None."""
    res = []
    for s in sizes:
        g = None
        ok = True
        try:
            g = arm.capture(xs[s], outs[s], s, calls)
        except Exception as e:  # pragma: no cover - depends on the arm
            ok = False
            print(f"graph capture of {s} bytes failed on this rank: {e}", file=sys.stderr)
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        us = -1.0
        if bool(flag.item()):
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
        del g  # graphs holding NCCL calls go before the process group does
        torch.cuda.synchronize()
        res.append(us)
    maxed = _max_over_ranks(res)
    return [None if v < 0 else v for v in maxed]


def timed_e2e(arm, xs, outs, sizes, steps, warmup):
    """Same sweep through the public API, with every input copied in from
    pinned host memory and every result read back to the host each step."""
    hx = {s: xs[s].cpu().pin_memory() for s in sizes}
    ho = {s: torch.empty(s // 2, dtype=torch.bfloat16).pin_memory() for s in sizes}

    def step():
        for s in sizes:
            xs[s].copy_(hx[s], non_blocking=True)
            r = arm.step_one(xs[s], outs[s], s)
            ho[s].copy_(r, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(max(1, warmup)):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    return _max_over_ranks([start.elapsed_time(end)])[0]


def verify(arm, sizes, rank, world):
    """The timed op really reduces: compare one mid-size message with NCCL."""
    s = min(sizes, key=lambda v: abs(v - (1 << 20)))
    torch.manual_seed(1234 + rank)
    x = torch.randn(s // 2, dtype=torch.bfloat16, device="cuda")
    ref = x.float()
    dist.all_reduce(ref)
    got = arm.step_one(x.clone(), torch.empty_like(x), s).float()
    ok = torch.allclose(got, ref, rtol=1e-2, atol=1e-2 * world)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def main():
    args = parse_args()
    sizes = [int(v) for v in args.sizes.split(",")] if args.sizes else SIZES
    if args.impl == "reference":
        try:
            import vllm  # noqa: F401
        except Exception as e:  # pragma: no cover - depends on the image
            print(json.dumps({"impl": "reference", "unavailable": f"vllm import failed: {e}"}))
            return 0
    rank, world, local = setup(args.gpus)
    arm = None
    try:
        try:
            arm = OursArm(local, sizes) if args.impl == "ours" else ReferenceArm(local, sizes)
        except Exception as e:
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference",
                                      "unavailable": f"{type(e).__name__}: {e}".splitlines()[0]}))
                return 0
            raise
        from numa_allreduce_b200.utils.timing import busbw_gbs, clocks_ok, pci_bus_id

        xs, outs = {}, {}
        for s in sizes:
            g = torch.Generator(device="cuda").manual_seed(rank)
            xs[s] = torch.randn(s // 2, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
            outs[s] = torch.empty_like(xs[s])
        bus = [None] * world
        dist.all_gather_object(bus, pci_bus_id(local))
        ok = verify(arm, sizes, rank, world)
        total_ms, p50_us, clocks, launches = timed_sweep(arm, xs, outs, sizes, args.steps, args.warmup,
                                                         rank, bus)
        e2e_ms = None if args.no_e2e else timed_e2e(arm, xs, outs, sizes, args.steps, min(args.warmup, 2))
        graph_us = None if args.no_graph else timed_graph(arm, xs, outs, sizes)
        bytes_per_step = sum(sizes)
        ms_per_step = total_ms / args.steps
        value = world * bytes_per_step / (ms_per_step / 1e3) / 1e9
        if rank == 0:
            sweep = [{"bytes": s, "p50_us": round(t, 2),
                      "busbw_gbs": round(busbw_gbs(s, t / 1e6, world), 1),
                      "algbw_gbs": round(s / (t / 1e6) / 1e9, 1), "algo": arm.algos[s]}
                     for s, t in zip(sizes, p50_us)]
            if graph_us is not None:
                for row, t in zip(sweep, graph_us):
                    row["graph_us"] = None if t is None else round(t, 2)
                    row["graph_busbw_gbs"] = None if t is None else round(busbw_gbs(row["bytes"], t / 1e6, world), 1)
            line = {
                "metric": METRIC,
                "value": round(value, 2),
                "unit": "GB/s",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": round(ms_per_step, 4),
                "higher_is_better": True,
                "scaling": "weak",
                "vs_baseline": None,
                "dtype": "bf16",
                "data": "synthetic: N(0,1) bf16, torch seed = rank",
                "impl": arm.name,
                "config": {
                    "model": "allreduce sweep: 17 contiguous 1-D bf16 messages, 4 KiB..256 MiB per rank",
                    "global_batch": len(sizes) * world,
                    "seq_len": bytes_per_step // 2,
                    "parallelism": f"allreduce over {world} GPU{'s' if world > 1 else ''} (one process per GPU)",
                    "value_definition": "n_gpus * bytes per rank per step / device time per step (aggregate algbw)",
                    "l2": "inputs larger than L2: a step touches 512 MiB per rank; each buffer is re-read only "
                          "after >256 MiB of other traffic",
                    "timing": "CUDA events on the launching stream, max over ranks; per-size p50 over steps; "
                              "sweep[].graph_us: per call, 10 calls replayed from one CUDA graph (after the "
                              "timed region, not part of value)",
                },
                "sweep": sweep,
                "sweep_busbw_gbs": round(busbw_gbs(bytes_per_step, ms_per_step / 1e3, world), 1),
                "verified_vs_nccl": ok,
            }
            if clocks is not None:
                line["clocks"] = clocks
                line["clocks_ok"] = clocks_ok(clocks)
            if e2e_ms is not None:
                line["e2e"] = {"value": round(world * bytes_per_step / (e2e_ms / args.steps / 1e3) / 1e9, 2),
                               "unit": "GB/s", "h2d_bytes_per_step": bytes_per_step,
                               "d2h_bytes_per_step": bytes_per_step,
                               "ms_per_step": round(e2e_ms / args.steps, 3)}
            line["gpu_launches"] = launches
            print(json.dumps(line), flush=True)
        return 0
    except Exception:
        traceback.print_exc()
        return 1
    finally:
        if arm is not None:
            try:
                torch.cuda.synchronize()
                arm.close()
            except Exception:
                traceback.print_exc()
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
