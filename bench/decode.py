#!/usr/bin/env python3
"""TP decode of a Llama-3-70B-shaped model in one CUDA graph.

hidden 8192, 80 layers, 64 q / 8 kv heads, head_dim 128, intermediate 28672,
random N(0, 0.02) bf16 weights, synthetic KV cache with 1024 tokens of
context, batch 1 / 8 / 32. Both variants of LlamaTPDecoder (this library's
fused path and the cuBLAS + NCCL + separate-norm baseline) are captured as
one CUDA graph per decode step; per-token latency is the replay time, max
over ranks. Launch one process per GPU:

    python -m torch.distributed.run --nproc-per-node 8 bench/decode.py
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from numa_allreduce_b200 import NumaAwareAllReduce  # noqa: E402
from numa_allreduce_b200.models.llama_tp import LlamaConfig, LlamaTPDecoder  # noqa: E402


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--batches", default="1,8,32")
    p.add_argument("--context", type=int, default=1024)
    p.add_argument("--layers", type=int, default=80)
    p.add_argument("--model", default="70b", choices=["70b", "8b", "tiny"])
    p.add_argument("--impls", default="fused,baseline")
    p.add_argument("--attention", default="tc", choices=["tc", "simt"])
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--shard-as", type=int, default=None,
                   help="single GPU: decode one rank's shard of an N-way TP model (no allreduce)")
    p.add_argument("--out", default=None)
    return p.parse_args()


def time_graph(model, reps):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            model.step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        model.step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    del g
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=600),
                            device_id=torch.device("cuda", local))
    cfg = {"70b": LlamaConfig.llama3_70b, "8b": LlamaConfig.llama3_8b, "tiny": LlamaConfig.tiny}[args.model]()
    cfg.layers = args.layers
    comm = NumaAwareAllReduce(dist.group.WORLD, device=local, fused_bytes=32 << 20)
    rows = []
    for B in [int(b) for b in args.batches.split(",")]:
        model = LlamaTPDecoder(cfg, comm, batch=B, context=args.context, shard_of=args.shard_as,
                               attention=args.attention)
        model.tokens.copy_(torch.arange(B, device="cuda") * 7 + 3)
        row = {"batch": B, "world_size": world, "context": args.context, "layers": cfg.layers,
               "weight_gb_per_rank": round(model.weight_bytes() / 1e9, 2)}
        finals = {}
        for impl in args.impls.split(","):
            model.impl = impl
            ms = time_graph(model, args.reps)
            model.step()
            torch.cuda.synchronize()
            finals[impl] = model.x.float().clone()
            row[f"{impl}_ms_per_token"] = round(ms, 4)
            row[f"{impl}_tokens_per_s"] = round(B / (ms / 1e3), 1)
        if "fused" in finals and "baseline" in finals:
            d = (finals["fused"] - finals["baseline"]).norm() / finals["baseline"].norm()
            row["rel_diff_final_hidden"] = float(d)
            row["speedup"] = round(row["baseline_ms_per_token"] / row["fused_ms_per_token"], 3)
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
        del model
        torch.cuda.empty_cache()
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            json.dump(rows, f, indent=1)
    torch.cuda.synchronize()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
