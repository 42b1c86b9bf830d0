#!/usr/bin/env python3
"""Accuracy of the TP decode step with depth, against fp32.

On one GPU, builds one rank's shard of the Llama-3-70B TP-8 decoder (the
same per-GPU shapes; ``--shard-of 8``), random-init weights N(0, 0.02), a
synthetic KV cache of ``--context`` tokens, and runs one decode step three
ways on the same weights and cache:

    fused     this library's kernels (tcgen05 GEMMs with the SwiGLU epilogue,
              fused RoPE + attention, fused residual + RMSNorm)
    baseline  cuBLAS GEMMs + the two-launch RoPE/attention + torch RMSNorm
    fp32      PyTorch in fp32 from the same bf16 weights and cache

and reports, per layer, the relative error ||h - h_fp32|| / ||h_fp32|| of the
residual stream for the two bf16 paths, and between them.

    python bench/decode_accuracy.py [--layers 80] [--batch 1] [--context 1024]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from numa_allreduce_b200.models.llama_tp import LlamaConfig, LlamaTPDecoder  # noqa: E402


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a - b).norm() / b.norm()).item()


def depth_errors(layers: int, batch: int, context: int, shard_of: int = 8, seed: int = 0) -> dict:
    cfg = LlamaConfig.llama3_70b()
    cfg.layers = layers
    m = LlamaTPDecoder(cfg, None, batch=batch, context=context, shard_of=shard_of, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    m.tokens.copy_(torch.randint(1, cfg.vocab, (batch,), generator=g, device="cuda"))
    ref = m.reference_step_fp32()
    traces = {}
    for impl in ("baseline", "fused"):
        m.impl = impl
        m.reset_position()
        t: list = []
        m.step(trace=t)
        torch.cuda.synchronize()
        traces[impl] = t
    per_layer = []
    for i in range(layers):
        per_layer.append({"layer": i + 1, "fused_vs_fp32": rel(traces["fused"][i], ref[i]),
                          "baseline_vs_fp32": rel(traces["baseline"][i], ref[i]),
                          "fused_vs_baseline": rel(traces["fused"][i], traces["baseline"][i])})
    return {"layers": layers, "batch": batch, "context": context, "shard_of": shard_of, "per_layer": per_layer}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--layers", type=int, default=80)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--context", type=int, default=1024)
    p.add_argument("--out", default=None)
    a = p.parse_args()
    torch.cuda.set_device(0)
    res = depth_errors(a.layers, a.batch, a.context)
    last = res["per_layer"][-1]
    print(json.dumps({k: v for k, v in res.items() if k != "per_layer"} | {"last": last}), flush=True)
    for row in res["per_layer"]:
        if row["layer"] in (1, 2, 4, 8, 16, 32, 64, 80) or row["layer"] == a.layers:
            print(json.dumps(row), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
