"""Llama-style decoder stack for decode over the quantized path.

Mirrors the reference caller Libraries/MLXLLM/Models/Llama.swift:10-127:
    h = x + o_proj(attn(rms_norm(x)))            (LlamaAttention, :49-80)
    out = h + down(silu(gate(rms(h))) * up(rms(h)))  (LlamaMLP, :96-99)
with every linear an MLX affine-quantized QuantizedLinear.  q/k/v are fused
into one column-parallel projection and gate/up into another (the fused
gate||up of SwitchLayers.swift:186-237 applied to a dense MLP), and o_proj /
down_proj are row-parallel with an all-reduce under tensor parallelism
(MLXDistributedTP ShardingPlan.llama, ShardingPlans+Llama.swift:40-50).

Weights are random-init (seeded): the reference loads checkpoints; the
benchmark has no network.  The whole decode step is a fixed sequence of
kernel launches on preallocated buffers, so it is captured once in a CUDA
graph and replayed per token.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from . import fast, ops


@dataclass
class LlamaConfig:
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    n_layers: int = 32
    rope_theta: float = 500000.0
    eps: float = 1e-5
    group_size: int = 64
    bits: int = 4


class QuantLinear:
    """(wq, scales, biases) of one quantized linear, in MLX layout."""

    def __init__(self, wq, scales, biases, group_size, bits):
        self.wq, self.scales, self.biases = wq, scales, biases
        self.group_size, self.bits = group_size, bits

    @property
    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.wq, self.scales, self.biases))

    def __call__(self, x, out=None):
        return ops.quantized_mm(x, self.wq, self.scales, self.biases, group_size=self.group_size,
                                bits=self.bits, out=out)

    def fused_swiglu(self, gate_up, residual=None, out=None):
        """silu(gate) * up -> matmul -> [+ residual], one kernel (decode, M <= 32)."""
        return ops.quantized_mm_swiglu(gate_up, self.wq, self.scales, self.biases, group_size=self.group_size,
                                       bits=self.bits, residual=residual, out=out)

    def fused(self, x, norm_weight=None, eps=1e-5, residual=None, out=None):
        """x -> [RMSNorm] -> matmul -> [+ residual], one kernel (decode, M <= 32)."""
        return ops.quantized_mm_fused(x, self.wq, self.scales, self.biases, group_size=self.group_size,
                                      bits=self.bits, norm_weight=norm_weight, eps=eps, residual=residual, out=out)


def shard_rows(t: torch.Tensor, rank: int, world: int, segments: List[int]) -> torch.Tensor:
    """Column-parallel slice (AllToShardedLinear, LinearLayers.swift:59-105): each
    output segment (e.g. q | k | v) is split into `world` equal row blocks and
    rank r keeps block r of every segment."""
    parts, start = [], 0
    for seg in segments:
        if seg % world:
            raise ValueError(f"segment {seg} not divisible by {world}")
        blk = seg // world
        parts.append(t[start + rank * blk: start + (rank + 1) * blk])
        start += seg
    return torch.cat(parts, 0).contiguous()


def shard_k(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row-parallel slice along K (ShardedToAllLinear, LinearLayers.swift:161-190) of a
    packed weight (last dim K*bits/32 words) or its scales / biases (last dim
    K/g): rank r keeps the r-th of `world` equal blocks, i.e. whole groups."""
    n = t.shape[-1]
    if n % world:
        raise ValueError(f"K blocks {n} not divisible by {world}")
    blk = n // world
    return t[..., rank * blk:(rank + 1) * blk].contiguous()


class LlamaLayerWeights:
    def __init__(self, cfg: LlamaConfig, dev, gen, rank: int = 0, world: int = 1):
        H, D, Hq, Hkv, F = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn
        g, b = cfg.group_size, cfg.bits

        def rnd(n, k):
            return (torch.randn(n, k, device=dev, generator=gen) * 0.02).bfloat16()

        def q(w):
            return ops.quantized(w, group_size=g, bits=b)

        # column-parallel: fused q | k | v and gate | up, quantized whole then row-sliced
        wqkv = q(rnd((Hq + 2 * Hkv) * D, H))
        segs = [Hq * D, Hkv * D, Hkv * D]
        self.qkv = QuantLinear(*[shard_rows(t, rank, world, segs) for t in wqkv], g, b)
        wgu = q(rnd(2 * F, H))
        self.gate_up = QuantLinear(*[shard_rows(t, rank, world, [F, F]) for t in wgu], g, b)
        # row-parallel: o_proj and down_proj sliced along K at group granularity
        wo = q(rnd(H, Hq * D))
        self.o = QuantLinear(*[shard_k(t, rank, world) for t in wo], g, b)
        wd = q(rnd(H, F))
        self.down = QuantLinear(*[shard_k(t, rank, world) for t in wd], g, b)
        self.norm1 = (1.0 + 0.1 * torch.randn(H, device=dev, generator=gen)).bfloat16()
        self.norm2 = (1.0 + 0.1 * torch.randn(H, device=dev, generator=gen)).bfloat16()

    @property
    def nbytes(self):
        return self.qkv.nbytes + self.gate_up.nbytes + self.o.nbytes + self.down.nbytes


class LlamaDecoder:
    """Decoder stack with per-layer bf16 KV caches [B, Hkv/P, max_len, D]."""

    def __init__(self, cfg: LlamaConfig, batch: int, max_len: int, dev, seed: int = 0,
                 rank: int = 0, world: int = 1, all_sum=None, cache_fill: int = 0, fused: bool = True,
                 group=None):
        if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.ffn % world:
            raise ValueError("heads / ffn not divisible by the TP size")
        self.cfg, self.B, self.max_len, self.dev = cfg, batch, max_len, dev
        self.rank, self.world, self.all_sum = rank, world, all_sum
        # group (distributed.Group): with fused=True under TP, o_proj / down_proj run as one
        # GEMV + all-reduce + residual kernel per rank (vmlx_tp_quantized_matmul_all_sum)
        self.group = group
        if all_sum is None and group is not None:
            self.all_sum = group.all_sum
        # fused: RMSNorm folded into the q/k/v and gate/up GEMVs (x staged normalised), and at TP=1
        # the residual adds folded into the o_proj / down_proj GEMVs (in place on x)
        # (decode rows 1-4 run the GEMV kernels that carry the fusions; from 5 rows the linears
        # run on the tensor-core GEMM and the norms / adds as their own kernels)
        self.fused = fused and batch <= 4
        self.hq, self.hkv, self.ffn = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.ffn // world
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.layers = [LlamaLayerWeights(cfg, dev, gen, rank, world) for _ in range(cfg.n_layers)]
        # KV caches: positions [0, cache_fill) hold random keys / values (the
        # benchmark's "4096 random tokens"), the decode step appends at `pos`.
        kv_gen = torch.Generator(device=dev).manual_seed(seed + 1)
        self.k_cache, self.v_cache = [], []
        for _ in range(cfg.n_layers):
            k = torch.zeros(batch, self.hkv, max_len, cfg.head_dim, dtype=torch.bfloat16, device=dev)
            v = torch.zeros_like(k)
            if cache_fill:
                k[:, :, :cache_fill].normal_(generator=kv_gen)
                v[:, :, :cache_fill].normal_(generator=kv_gen)
            self.k_cache.append(k)
            self.v_cache.append(v)
        D = cfg.head_dim
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.h = torch.empty(batch, cfg.hidden, **bf)
        self.qkv_buf = torch.empty(batch, (self.hq + 2 * self.hkv) * D, **bf)
        self.q = torch.empty(batch, self.hq, D, **bf)
        self.attn = torch.empty(batch, self.hq, D, **bf)
        self.proj = torch.empty(batch, cfg.hidden, **bf)
        self.gu = torch.empty(batch, 2 * self.ffn, **bf)
        self.act = torch.empty(batch, self.ffn, **bf)
        self.ws = torch.zeros(max(fast.sdpa_workspace_bytes(batch, self.hq, max_len, D), 4),
                              dtype=torch.uint8, device=dev)

    @property
    def weight_bytes(self):
        return sum(l.nbytes for l in self.layers)

    def _reduce(self, t):
        if self.world > 1:
            self.all_sum(t)

    def step(self, x: torch.Tensor, pos: int) -> torch.Tensor:
        """One decode step for B tokens at cache position `pos` (in place on x)."""
        cfg = self.cfg
        fused, tp = self.fused, self.world > 1
        tp_fused = fused and tp and self.group is not None
        for i, L in enumerate(self.layers):
            if fused:
                L.qkv.fused(x, norm_weight=L.norm1, eps=cfg.eps, out=self.qkv_buf)
            else:
                fast.rms_norm(x, L.norm1, cfg.eps, out=self.h)
                L.qkv(self.h, out=self.qkv_buf)
            fast.rope_qkv(self.qkv_buf, self.k_cache[i], self.v_cache[i], self.hq, self.hkv, pos,
                          base=cfg.rope_theta, q_out=self.q)
            fast.sdpa_decode(self.q, self.k_cache[i], self.v_cache[i], pos + 1, workspace=self.ws,
                             out=self.attn)
            if fused and not tp:
                L.o.fused(self.attn.view(self.B, -1), residual=x, out=x)
            elif tp_fused:
                self.group.quantized_matmul_all_sum(self.attn.view(self.B, -1), L.o, residual=x, out=x)
            else:
                L.o(self.attn.view(self.B, -1), out=self.proj)
                self._reduce(self.proj)
                fast.add(x, self.proj, out=x)
            if fused:
                L.gate_up.fused(x, norm_weight=L.norm2, eps=cfg.eps, out=self.gu)
            else:
                fast.rms_norm(x, L.norm2, cfg.eps, out=self.h)
                L.gate_up(self.h, out=self.gu)
            if fused and not tp:  # SwiGLU fused into the down GEMV's x staging
                L.down.fused_swiglu(self.gu, residual=x, out=x)
            elif tp_fused:
                self.group.quantized_matmul_all_sum(self.gu, L.down, residual=x, out=x, swiglu=True)
            else:
                fast.silu_mul(self.gu, out=self.act)
                L.down(self.act, out=self.proj)
                self._reduce(self.proj)
                fast.add(x, self.proj, out=x)
        return x

    # ---- CUDA-graph decode (the public per-token call) ----
    @property
    def launches_per_step(self):
        # per layer: 4 GEMV, rope, sdpa (one kernel, combine fused); unfused: + silu_mul + 2 rms_norm;
        # TP: + 2 all-reduce + 2 add unless the row-parallel GEMVs carry the all-reduce and residual
        tp_fused = self.world > 1 and self.fused and self.group is not None
        n = 6 + (0 if self.fused and (self.world == 1 or tp_fused) else 1) + (0 if self.fused else 2)
        if self.world > 1 and not tp_fused:
            n += 4
        elif not self.fused:
            n += 2
        return self.cfg.n_layers * n

    def capture(self, x: torch.Tensor, pos: int, stream=None) -> "torch.cuda.CUDAGraph":
        """Capture step(x, pos) on `stream` into a CUDA graph (x is the graph's
        input/output buffer).  Replaying it performs one decode step."""
        stream = stream or torch.cuda.Stream(self.dev)
        self._gx = x
        x_save = x.clone()
        with torch.cuda.stream(stream):
            self.step(x, pos)  # warm-up outside capture (loads kernels, sets attributes)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self.step(x, pos)
            x.copy_(x_save)
        torch.cuda.synchronize()
        self._graph, self._gstream = g, stream
        return g

    def decode(self, x_host: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step from host memory: copy the token states in, replay the
        captured step, copy the result back (asynchronously on the capture stream)."""
        if getattr(self, "_graph", None) is None:
            raise RuntimeError("call capture() first")
        st = self._gstream
        with torch.cuda.stream(st):
            self._gx.copy_(x_host, non_blocking=True)
            self._graph.replay()
            out = torch.empty_like(x_host, pin_memory=True) if out is None else out
            out.copy_(self._gx, non_blocking=True)
        return out
