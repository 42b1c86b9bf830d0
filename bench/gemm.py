#!/usr/bin/env python3
"""tcgen05 GEMM against cuBLAS on the decode shapes of Llama-3-70B at TP 8.

``y[T, N] = x[T, K] @ wt[N, K].T`` in bf16, fp32 accumulation, for the
projections one rank runs per layer (qkv 1280x8192, o 8192x1024, gate|up
7168x8192, down 8192x3584, lm_head 16128x8192) and token counts 1..512;
`--shapes 8b_qkv,8b_o,8b_gate_up,8b_down` gives the Llama-3-8B TP-8 ones.
Weights rotate over enough copies to exceed the 126 MB L2, so every call
streams its weight from HBM; each variant is timed as `--calls` launches
captured in one CUDA graph (launch overhead as in a decode step), CUDA
events around the replays. Reports microseconds per call and the weight
streaming rate (weight bytes / time), for the row-major weight and for the
tiled layout of `pack_weight` (16 KB contiguous per weight tile). Back-to-back launches of this
library's GEMM overlap through programmatic dependent launch (the next
call's weight prefetch starts during the previous call); `--no-pdl`
measures them serialised like the cuBLAS calls.

    python bench/gemm.py [--tokens 1,8,32] [--out gemm.json]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from numa_allreduce_b200.ops import _ext  # noqa: E402
from numa_allreduce_b200.ops.gemm import gemm, pack_weight  # noqa: E402

SHAPES = {"qkv": (1280, 8192), "o": (8192, 1024), "gate_up": (7168, 8192), "down": (8192, 3584),
          "lm_head": (16128, 8192),
          # Llama-3-8B at TP 8 (the fused layer tail's down projection is 8b_down)
          "8b_qkv": (768, 4096), "8b_o": (4096, 512), "8b_gate_up": (3584, 4096), "8b_down": (4096, 1792)}
DEFAULT_SHAPES = "qkv,o,gate_up,down,lm_head"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", default="1,8,16,32,64,128,512")
    p.add_argument("--shapes", default=DEFAULT_SHAPES, help="comma list of " + ",".join(SHAPES))
    p.add_argument("--calls", type=int, default=20)
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--splits", type=int, default=0, help="force a split count (0: the heuristic)")
    p.add_argument("--no-pdl", action="store_true", help="launch the GEMMs without programmatic dependent launch")
    p.add_argument("--split-sweep", action="store_true",
                   help="time the packed-weight GEMM at every split count 1..16 and report the best against "
                        "the heuristic's choice")
    p.add_argument("--out", default=None)
    return p.parse_args()


def time_graph(fn, calls, reps):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(2):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(calls):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        best = min(best, a.elapsed_time(b) * 1e3 / calls)
    del g
    return best


def main():
    a = parse()
    if a.no_pdl:
        os.environ["NAB_GEMM_PDL"] = "0"  # read at the first GEMM launch
    ops = _ext.load()
    dev = torch.device("cuda")
    rows = []
    for name in a.shapes.split(","):
        N, K = SHAPES[name]
        copies = max(2, (256 << 20) // (N * K * 2) + 1)
        ws = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
        wps = [pack_weight(w) for w in ws]
        for T in [int(t) for t in a.tokens.split(",")]:
            x = torch.randn(T, K, device=dev, dtype=torch.bfloat16)
            y = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
            splits = a.splits or int(ops.gemm_splits(T, N, K))
            if a.split_sweep:
                kb = K // 64
                times = {}
                for sp in range(1, 17):
                    per = -(-kb // sp)
                    if -(-kb // per) != sp:  # a split without work: not a launchable count
                        continue
                    times[sp] = round(time_graph(lambda i: gemm(x, wps[i % copies], out=y, splits=sp), a.calls,
                                                 a.reps), 2)
                best = min(times, key=times.get)
                row = {"shape": name, "T": T, "auto_splits": splits, "auto_us": times.get(splits),
                       "best_splits": best, "best_us": times[best], "times_us": times}
                rows.append(row)
                print(json.dumps(row), flush=True)
                continue
            ref = F.linear(x, ws[0]).float()
            err = (gemm(x, ws[0], out=y, splits=splits).float() - ref).abs().max().item()
            err_p = (gemm(x, wps[0], out=y, splits=splits).float() - ref).abs().max().item()
            ours = time_graph(lambda i: gemm(x, ws[i % copies], out=y, splits=splits), a.calls, a.reps)
            packed = time_graph(lambda i: gemm(x, wps[i % copies], out=y, splits=splits), a.calls, a.reps)
            cub = time_graph(lambda i: torch.matmul(x, ws[i % copies].t(), out=y), a.calls, a.reps)
            wbytes = N * K * 2
            row = {"shape": name, "T": T, "N": N, "K": K, "splits": splits, "ours_us": round(ours, 2),
                   "packed_us": round(packed, 2), "packed_tbs": round(wbytes / packed / 1e6, 2),
                   "cublas_us": round(cub, 2), "ours_tbs": round(wbytes / ours / 1e6, 2),
                   "cublas_tbs": round(wbytes / cub / 1e6, 2), "speedup": round(cub / ours, 3),
                   "max_abs_err": max(err, err_p)}
            rows.append(row)
            print(json.dumps(row), flush=True)
        del ws, wps
        torch.cuda.empty_cache()
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
