#!/usr/bin/env python3
"""Decode attention of one TP-8 rank of Llama-3-70B (8 query heads, 1 kv
head, head_dim 128) for batch 1..32 and a 1024-token context.

Times `--calls` launches captured in one CUDA graph, each on another layer's
KV cache (more bytes than the 126 MB L2 across the rotation), CUDA events
around the replays:

    rope_attention     this library: RoPE + KV append + attention, one launch
    decode_attention   this library: attention only (q already rotated)
    *_tc               the same on the tensor cores (tcgen05 scores and
                       output, TMA-staged K/V chunks of 128 positions)
    sdpa               torch scaled_dot_product_attention (GQA expanded)

    python bench/attention.py [--batches 1,8,32] [--context 1024]
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
    p = argparse.ArgumentParser()
    p.add_argument("--batches", default="1,8,32")
    p.add_argument("--context", type=int, default=1024)
    p.add_argument("--hq", type=int, default=8)
    p.add_argument("--hkv", type=int, default=1)
    p.add_argument("--calls", type=int, default=40)
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--splits", type=int, default=0)
    a = p.parse_args()
    ops = _ext.load()
    D, Hq, Hkv = 128, a.hq, a.hkv
    Lmax = ((a.context + 1 + 63) // 64) * 64
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float64) / D))
    ang = torch.arange(Lmax, device="cuda", dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()
    pos = torch.tensor([a.context], device="cuda", dtype=torch.int32)
    for B in [int(x) for x in a.batches.split(",")]:
        kv_bytes = 2 * B * Hkv * (a.context + 1) * D * 2
        copies = max(2, min(a.calls, (512 << 20) // (2 * B * Hkv * Lmax * D * 2) + 1))
        ks = [torch.randn(B, Hkv, Lmax, D, device="cuda", dtype=torch.bfloat16) for _ in range(copies)]
        vs = [torch.randn(B, Hkv, Lmax, D, device="cuda", dtype=torch.bfloat16) for _ in range(copies)]
        qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        splits = a.splits or int(ops.attention_splits(B, Hkv, a.context + 1))
        t_rope = time_graph(lambda i: ops.rope_attention(qkv, cos, sin, pos, ks[i % copies], vs[i % copies], out,
                                                         Hq, Hkv, splits), a.calls, a.reps)
        t_attn = time_graph(lambda i: ops.decode_attention(q, ks[i % copies], vs[i % copies], pos, out, splits),
                            a.calls, a.reps)
        sp_tc = a.splits or int(ops.attention_splits_tc(B, Hkv, a.context + 1))
        t_rope_tc = time_graph(lambda i: ops.rope_attention_tc(qkv, cos, sin, pos, ks[i % copies], vs[i % copies],
                                                               out, Hq, Hkv, sp_tc), a.calls, a.reps)
        t_attn_tc = time_graph(lambda i: ops.decode_attention_tc(q, ks[i % copies], vs[i % copies], pos, out,
                                                                 sp_tc), a.calls, a.reps)
        L = a.context + 1

        def sdpa(i):
            k = ks[i % copies][:, :, :L].repeat_interleave(Hq // Hkv, dim=1)
            v = vs[i % copies][:, :, :L].repeat_interleave(Hq // Hkv, dim=1)
            return F.scaled_dot_product_attention(q.unsqueeze(2), k, v)

        t_sdpa = time_graph(sdpa, a.calls, a.reps)
        row = {"batch": B, "context": a.context, "splits": splits, "kv_mb": round(kv_bytes / 1e6, 2),
               "rope_attention_us": round(t_rope, 2), "decode_attention_us": round(t_attn, 2),
               "sdpa_us": round(t_sdpa, 2), "attn_tbs": round(kv_bytes / t_attn / 1e6, 3),
               "splits_tc": sp_tc, "rope_attention_tc_us": round(t_rope_tc, 2),
               "decode_attention_tc_us": round(t_attn_tc, 2), "attn_tc_tbs": round(kv_bytes / t_attn_tc / 1e6, 3)}
        print(json.dumps(row), flush=True)
        del ks, vs
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
