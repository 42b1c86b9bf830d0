#!/usr/bin/env python3
"""Where the time of one TP decode step goes, on one GPU.

Builds one rank's shard of the Llama-3-70B TP-8 decoder (same per-GPU
shapes, no allreduce) and times CUDA-graph replays of the full step and of
ablated steps in which one group of kernels is replaced by nothing:

    full          the step as decoded
    no_attention  without RoPE/KV append and attention
    no_norm       without the residual + RMSNorm kernels
    gemm_only     only the projections (and the embedding / argmax)

The difference to `full` is the marginal cost of a group inside the graph
(overlap included). Analysis only: an ablated step computes garbage.

    python bench/decode_breakdown.py [--batch 1] [--layers 80]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from numa_allreduce_b200.models import llama_tp  # noqa: E402
from numa_allreduce_b200.models.llama_tp import LlamaConfig, LlamaTPDecoder  # noqa: E402


class _Skip:
    """Proxy over the extension's ops that turns the named ones into no-ops."""

    def __init__(self, ops, skip):
        self._ops, self._skip = ops, set(skip)

    def __getattr__(self, name):
        if name in self._skip:
            return lambda *a, **k: None
        return getattr(self._ops, name)


def time_step(model, reps):
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
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / reps


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--layers", type=int, default=80)
    p.add_argument("--tp", type=int, default=8)
    p.add_argument("--context", type=int, default=1024)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--impl", default="fused")
    p.add_argument("--attention", default="tc", choices=["tc", "simt"])
    a = p.parse_args()
    cfg = LlamaConfig.llama3_70b()
    cfg.layers = a.layers
    model = LlamaTPDecoder(cfg, None, batch=a.batch, context=a.context, impl=a.impl, shard_of=a.tp,
                           attention=a.attention)
    real_ops = model.ops
    real_norm = llama_tp.rmsnorm_residual
    out = {"batch": a.batch, "layers": a.layers, "tp": a.tp, "impl": a.impl, "attention": a.attention}
    attn_ops = ["rope_append", "decode_attention", "rope_attention", "rope_attention_tc"]
    variants = {
        "full": ([], False),
        "no_attention": (attn_ops, False),
        "no_norm": ([], True),
        "gemm_only": (attn_ops + ["silu_mul"], True),
    }
    for name, (skip, no_norm) in variants.items():
        model.ops = _Skip(real_ops, skip)
        llama_tp.rmsnorm_residual = (lambda *x, **k: None) if no_norm else real_norm
        out[f"{name}_ms"] = round(time_step(model, a.reps), 4)
    model.ops = real_ops
    llama_tp.rmsnorm_residual = real_norm
    per_layer = 1e3 / a.layers
    out["attention_us_per_layer"] = round((out["full_ms"] - out["no_attention_ms"]) * per_layer, 2)
    out["norms_us_per_layer"] = round((out["full_ms"] - out["no_norm_ms"]) * per_layer, 2)
    out["gemm_us_per_layer"] = round(out["gemm_only_ms"] * per_layer, 2)
    out["weight_gb"] = round(model.weight_bytes() / 1e9, 2)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
