"""Tensor-parallel Llama decoder for CUDA-graph decode.

Llama-3 architecture (GQA attention with rotary embeddings, SwiGLU MLP,
RMSNorm), sharded Megatron-style over the ranks: q/k/v and gate/up
projections are column-parallel, o_proj and down_proj row-parallel, so each
layer ends in two allreduces. Both are fused with the residual add and the
next RMSNorm:

* ``impl="fused"`` (this library): tcgen05 GEMMs on weights in the tiled
  layout (one contiguous 16 KB block per weight tile), launched as
  programmatic dependent launches so each weight stream starts during the
  kernel before; the gate|up GEMM applies SwiGLU in its epilogue; each
  row-parallel GEMM stores its output tiles into every rank's buffer over
  NVLink and a second kernel adds them with the residual and applies the
  next RMSNorm (above the fused slot size: the GEMM plus the fused
  allreduce + residual + RMSNorm kernel);
* ``impl="baseline"``: cuBLAS (``F.linear``) + NCCL ``all_reduce`` + residual
  add + ``F.rms_norm``, the unfused stack.

Attention (decode over a synthetic KV cache) uses this library's kernels in
both variants: the baseline as separate RoPE/KV-append and attention
launches, the fused variant as one launch that does both. Weights are random N(0, 0.02) (there is no
checkpoint), the KV cache random N(0, 1); every buffer a step touches is
static so the whole step is captured in one CUDA graph.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops import _ext
from ..ops.errors import check_enabled, check_kernels
from ..ops.fused import fused_allreduce_rmsnorm, rmsnorm_residual
from ..ops.gemm import gemm, gemm_allreduce_rmsnorm, gemm_swiglu, interleave_gate_up, pack_weight


@dataclass
class LlamaConfig:
    hidden: int = 8192
    layers: int = 80
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 28672
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @classmethod
    def llama3_70b(cls) -> "LlamaConfig":
        return cls()

    @classmethod
    def llama3_8b(cls) -> "LlamaConfig":
        return cls(hidden=4096, layers=32, heads=32, kv_heads=8, intermediate=14336)

    @classmethod
    def tiny(cls) -> "LlamaConfig":
        return cls(hidden=1024, layers=2, heads=16, kv_heads=8, intermediate=2048, vocab=4096)


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class LlamaTPDecoder:
    """One rank's shard of the model plus the static buffers of a decode step.

    Row-parallel tails use the fused GEMM + allreduce + norm whenever the
    output fits the communicator's fused slots (``fused_bytes``): the one-shot
    epilogue for a few tokens, the reduce-scatter epilogue (each token row to
    its owner rank, then a gather of the new residual rows) from 8 tokens per
    rank on. Larger outputs take this library's GEMM followed by its fused
    allreduce + residual + RMSNorm kernel. No library GEMM is on the path.

    Args:
        cfg: model shape.
        comm: this rank's :class:`~numa_allreduce_b200.NumaAwareAllReduce`
            (``None`` or world size 1 for a single GPU).
        batch: sequences decoded per step.
        context: tokens already in the (synthetic) KV cache; the step decodes
            position ``context``.
        impl: ``"fused"`` or ``"baseline"`` (see module docstring).
        shard_of: with a single GPU, build the shard of a ``shard_of``-way
            tensor-parallel model (same per-GPU shapes, no allreduce), to
            study one rank's kernels alone.
        attention: ``"tc"`` for the tensor-core decode attention (tcgen05
            scores and output per 128-position chunk), ``"simt"`` for the
            SIMT kernel; the fused variant only (the baseline uses the
            two-launch SIMT path).
    """

    def __init__(self, cfg: LlamaConfig, comm, batch: int, context: int, impl: str = "fused", seed: int = 0,
                 device: torch.device | str = "cuda", attn_splits: int | None = None, shard_of: int | None = None,
                 attention: str = "tc"):
        if impl not in ("fused", "baseline"):
            raise ValueError("impl must be 'fused' or 'baseline'")
        self.cfg, self.comm, self.impl = cfg, comm, impl
        self.device = torch.device(device)
        self.world = comm.world_size if comm is not None and not comm.disabled else 1
        self.rank = comm.rank if self.world > 1 else 0
        if shard_of is not None and self.world > 1 and shard_of != self.world:
            raise ValueError("shard_of is for a single GPU (or must equal the world size)")
        W = shard_of or self.world
        if cfg.heads % W or cfg.intermediate % W:
            raise ValueError("heads and intermediate size must divide by the world size")
        self.ops = _ext.load()
        D = cfg.head_dim
        self.Hq = cfg.heads // W
        self.Hkv = max(1, cfg.kv_heads // W)  # kv heads replicated when W > kv_heads
        self.tp = W
        self.I = cfg.intermediate // W
        self.B, self.ctx = batch, context
        self.Lmax = _round_up(context + 1, 64)
        H = cfg.hidden
        g = torch.Generator(device=self.device).manual_seed(1234 + self.rank + 7919 * seed)

        def w(rows, cols):
            return (torch.randn(rows, cols, generator=g, device=self.device, dtype=torch.bfloat16) * 0.02)

        qkv_rows = (self.Hq + 2 * self.Hkv) * D
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "wqkv": w(qkv_rows, H), "wo": w(H, self.Hq * D), "wgu": w(2 * self.I, H), "wd": w(H, self.I),
                "in_norm": torch.ones(H, device=self.device, dtype=torch.bfloat16),
                "post_norm": torch.ones(H, device=self.device, dtype=torch.bfloat16),
                "k": torch.randn(batch, self.Hkv, self.Lmax, D, generator=g, device=self.device,
                                 dtype=torch.bfloat16),
                "v": torch.randn(batch, self.Hkv, self.Lmax, D, generator=g, device=self.device,
                                 dtype=torch.bfloat16),
            })
        gv = torch.Generator(device=self.device).manual_seed(4321 + 7919 * seed)  # replicated tables
        self.embed = torch.randn(cfg.vocab, H, generator=gv, device=self.device, dtype=torch.bfloat16) * 0.02
        self.final_norm = torch.ones(H, device=self.device, dtype=torch.bfloat16)
        self.v_local = _round_up((cfg.vocab + W - 1) // W, 128)
        self.lm_head = w(self.v_local, H)
        # this library's GEMM reads weights in the tiled layout (one
        # contiguous 16 KB block of HBM per weight tile); built on first use
        # of the fused path
        self._packed: dict[tuple[int, str], object] = {}
        # rotary tables
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=self.device, dtype=torch.float64) / D))
        ang = torch.arange(self.Lmax, device=self.device, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()
        # static step buffers
        bf = dict(device=self.device, dtype=torch.bfloat16)
        self.tokens = torch.zeros(batch, device=self.device, dtype=torch.long)
        self.pos = torch.tensor([context], device=self.device, dtype=torch.int32)
        self.h = torch.empty(batch, H, **bf)
        self.x = torch.empty(batch, H, **bf)
        self.qkv = torch.empty(batch, qkv_rows, **bf)
        self.q = torch.empty(batch, self.Hq, D, **bf)
        self.attn = torch.empty(batch, self.Hq * D, **bf)
        self.gu = torch.empty(batch, 2 * self.I, **bf)
        self.act = torch.empty(batch, self.I, **bf)
        self.y = torch.empty(batch, H, **bf)
        self.logits = torch.empty(batch, self.v_local, **bf)
        if attention not in ("tc", "simt"):
            raise ValueError("attention must be 'tc' (tensor cores) or 'simt'")
        self.attention = attention
        self.splits = attn_splits or int(self.ops.attention_splits(batch, self.Hkv, context + 1))
        self.splits_tc = attn_splits or int(self.ops.attention_splits_tc(batch, self.Hkv, context + 1))
        self.gemm_splits = {}
        self.next_tokens = torch.zeros(batch, device=self.device, dtype=torch.long)
        self._gathered = torch.empty(W * batch * 2, device=self.device, dtype=torch.float32)

    # --------------------------------------------------------------- pieces --
    def _w(self, layer: int, key: str):
        """Weight `key` of `layer` (-1: lm_head) in the layout the variant reads."""
        wt = self.lm_head if layer < 0 else self.layers[layer][key]
        if self.impl == "baseline":
            return wt
        pw = self._packed.get((layer, key))
        if pw is None:
            # gate|up rows interleaved in 64-row blocks for the SwiGLU epilogue
            pw = self._packed[(layer, key)] = pack_weight(interleave_gate_up(wt) if key == "wgu" else wt)
        return pw

    def _proj(self, x, wt, out):
        if self.impl == "baseline":
            out.copy_(F.linear(x, wt))
        else:
            gemm(x, wt, out=out)
        return out

    def _row_parallel_tail(self, inp, layer: int, key: str, norm_w):
        """residual h += allreduce(inp @ W.T); x = rmsnorm(h) * norm_w."""
        eps = self.cfg.eps
        w_rows = self.layers[layer][key]  # row-major [out, in]
        if self.impl == "baseline":
            y = F.linear(inp, w_rows)
            if self.world > 1:
                dist.all_reduce(y)
            self.h.add_(y)
            self.x.copy_(F.rms_norm(self.h, (self.cfg.hidden,), norm_w, eps))
            return
        if self.world == 1:
            gemm(inp, self._w(layer, key), out=self.y)
            rmsnorm_residual(self.y, self.h, norm_w, eps, out=self.x)
        elif self.B * self.cfg.hidden * 2 <= self.comm.fused_bytes:
            # one-shot epilogue for few tokens, reduce-scatter epilogue from 8
            # tokens per rank on (both this library's tcgen05 GEMM)
            gemm_allreduce_rmsnorm(self.comm, inp, self._w(layer, key), self.h, norm_w, eps, out=self.x)
        else:
            # more rows than the fused slots hold: this library's GEMM, then its
            # fused allreduce + residual + RMSNorm
            gemm(inp, self._w(layer, key), out=self.y)
            fused_allreduce_rmsnorm(self.comm, self.y, self.h, norm_w, eps, out=self.x)

    def step(self, trace: list | None = None):
        """One decode step (graph-capturable): tokens -> next tokens. With
        ``trace`` (eager only) the residual stream after every layer is
        appended to it as fp32."""
        cfg, ops = self.cfg, self.ops
        torch.index_select(self.embed, 0, self.tokens, out=self.h)
        self.x.copy_(F.rms_norm(self.h, (cfg.hidden,), self.layers[0]["in_norm"], cfg.eps))
        for i, L in enumerate(self.layers):
            self._proj(self.x, self._w(i, "wqkv"), self.qkv)
            attn = self.attn.view(self.B, self.Hq, cfg.head_dim)
            if self.impl == "baseline":
                ops.rope_append(self.qkv, self.cos, self.sin, self.pos, self.q, L["k"], L["v"], self.Hq, self.Hkv)
                ops.decode_attention(self.q, L["k"], L["v"], self.pos, attn, self.splits)
            elif self.attention == "tc":
                ops.rope_attention_tc(self.qkv, self.cos, self.sin, self.pos, L["k"], L["v"], attn, self.Hq,
                                      self.Hkv, self.splits_tc)
            else:
                ops.rope_attention(self.qkv, self.cos, self.sin, self.pos, L["k"], L["v"], attn, self.Hq, self.Hkv,
                                   self.splits)
            self._row_parallel_tail(self.attn, i, "wo", L["post_norm"])
            if self.impl == "baseline":
                self._proj(self.x, self._w(i, "wgu"), self.gu)
                ops.silu_mul(self.gu, self.act)
            else:
                gemm_swiglu(self.x, self._w(i, "wgu"), out=self.act)
            nxt = self.layers[i + 1]["in_norm"] if i + 1 < len(self.layers) else self.final_norm
            self._row_parallel_tail(self.act, i, "wd", nxt)
            if trace is not None:
                trace.append(self.h.float().clone())
        self._proj(self.x, self._w(-1, "lm_head"), self.logits)
        val, idx = self.logits.float().max(dim=-1)
        if self.world > 1:
            mine = torch.stack([val, (idx + self.rank * self.v_local).float()], dim=-1).reshape(-1)
            dist.all_gather_into_tensor(self._gathered, mine)
            allv = self._gathered.view(self.world, self.B, 2)
            best = allv[:, :, 0].argmax(dim=0)
            self.next_tokens.copy_(allv[best, torch.arange(self.B, device=self.device), 1].long())
        else:
            self.next_tokens.copy_(idx)
        if check_enabled() and not torch.cuda.is_current_stream_capturing():
            check_kernels()
            if self.comm is not None:
                self.comm.check()
        return self.next_tokens

    def reset_position(self):
        self.pos.fill_(self.ctx)

    @torch.no_grad()
    def reference_step_fp32(self) -> list[torch.Tensor]:
        """The same decode step in fp32 PyTorch from the same (bf16) weights
        and KV cache, on one GPU (world size 1, or a ``shard_of`` shard):
        returns the residual stream after every layer. Positions before the
        current one come from the cache; the current position's k and v are
        this function's own (the cache is not written)."""
        if self.world != 1:
            raise ValueError("the fp32 reference runs on one GPU (world size 1 or shard_of)")
        cfg = self.cfg
        D, B, Hq, Hkv = cfg.head_dim, self.B, self.Hq, self.Hkv
        pos = int(self.pos.item())
        c, s = self.cos[pos], self.sin[pos]

        def rot(t):
            a, b = t[..., :D // 2], t[..., D // 2:]
            return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

        def norm(t, w):
            return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + cfg.eps) * w.float()

        h = self.embed.index_select(0, self.tokens).float()
        x = norm(h, self.layers[0]["in_norm"])
        out = []
        for i, L in enumerate(self.layers):
            qkv = x @ L["wqkv"].float().t()
            q = rot(qkv[:, :Hq * D].view(B, Hq, D))
            k_new = rot(qkv[:, Hq * D:(Hq + Hkv) * D].view(B, Hkv, D))
            v_new = qkv[:, (Hq + Hkv) * D:].view(B, Hkv, D)
            k = torch.cat([L["k"][:, :, :pos].float(), k_new[:, :, None]], dim=2)
            v = torch.cat([L["v"][:, :, :pos].float(), v_new[:, :, None]], dim=2)
            g = Hq // Hkv
            k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
            p = (torch.einsum("bhd,bhld->bhl", q, k) / math.sqrt(D)).softmax(-1)
            attn = torch.einsum("bhl,bhld->bhd", p, v).reshape(B, Hq * D)
            h = h + attn @ L["wo"].float().t()
            x = norm(h, L["post_norm"])
            gu = x @ L["wgu"].float().t()
            act = F.silu(gu[:, :self.I]) * gu[:, self.I:]
            h = h + act @ L["wd"].float().t()
            nxt = self.layers[i + 1]["in_norm"] if i + 1 < len(self.layers) else self.final_norm
            x = norm(h, nxt)
            out.append(h.clone())
        return out

    def weight_bytes(self) -> int:
        n = sum(t.numel() for L in self.layers for k, t in L.items() if k.startswith("w"))
        return 2 * (n + self.lm_head.numel())


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, length: int) -> torch.Tensor:
    """fp32 GQA decode attention: q [B, Hq, D], k/v [B, Hkv, Lmax, D]."""
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    kk = k[:, :, :length].float().repeat_interleave(Hq // Hkv, dim=1)
    vv = v[:, :, :length].float().repeat_interleave(Hq // Hkv, dim=1)
    s = torch.einsum("bhd,bhld->bhl", q.float(), kk) / math.sqrt(D)
    return torch.einsum("bhl,bhld->bhd", s.softmax(-1), vv)
