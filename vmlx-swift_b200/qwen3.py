"""Qwen3 dense decoder with a full greedy token loop (Qwen3-32B-shaped).

Mirrors the reference model Libraries/MLXLLM/Models/Qwen3.swift:15-245 and the generation
loop of Libraries/MLXLMCommon/Evaluate.swift:2505-2578 over this library's kernels:
    h = embed_tokens(ids)                                        (QuantizedEmbedding)
    per layer:  h += o_proj(attn(rope(q_norm(q)), rope(k_norm(k)), v))  with q|k|v = qkv(rms(h))
                h += down(silu(gate(rms(h))) * up(rms(h)))
    logits = lm_head(rms(h));  next = argMax(logits)             (ArgMaxSampler)
with every linear (and the embedding) an MLX affine-quantized matrix.  The decode step is
one CUDA graph: the token ids and the cache position live in device memory, the step reads
them, writes the sampled ids back and advances the position on the device, so the same
graph is replayed for every generated token (the reference re-evaluates a lazy graph per
token).

The prompt is prefilled with the same linears at M = batch x prompt rows (the tcgen05 GEMM)
and the per-head norms / RoPE / cache append of the decode kernel in its prefill mode;
prefill attention (causal, over the prompt) uses torch's scaled_dot_product_attention,
library code outside the decode path this package replaces.

Weights are random-init in the quantized domain (seeded): uniform 4-bit codes with per-group
bf16 scales and biases of the size a quantized N(0, 0.02) matrix has.  The bytes streamed per
token are those of the real model; there is no network for checkpoints.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from . import fast, ops
from .llama import QuantLinear


@dataclass
class Qwen3Config:
    hidden: int = 5120
    n_heads: int = 64
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 25600
    n_layers: int = 64
    vocab: int = 151936
    rope_theta: float = 1000000.0
    eps: float = 1e-6
    group_size: int = 64
    bits: int = 4


def random_quantized(n: int, k: int, group_size: int, bits: int, dev, gen, std: float = 0.02):
    """(w, scales, biases) of an [n, k] matrix drawn in the quantized domain: codes uniform in
    [0, 2^bits), scale ~ range of a group of N(0, std) values / (2^bits - 1), bias = -scale *
    2^(bits-1) (the group centred on zero)."""
    levels = (1 << bits) - 1
    w = torch.randint(-(1 << 31), 1 << 31, (n, k * bits // 32), device=dev, generator=gen, dtype=torch.int32)
    g = k // group_size
    spread = 5.0 * std * (0.8 + 0.4 * torch.rand(n, g, device=dev, generator=gen))
    scales = (spread / levels).bfloat16()
    biases = (-scales.float() * (1 << (bits - 1))).bfloat16()
    return w, scales, biases


class Qwen3Layer:
    def __init__(self, cfg: Qwen3Config, dev, gen):
        H, D, Hq, Hkv, F = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn
        g, b = cfg.group_size, cfg.bits
        self.qkv = QuantLinear(*random_quantized((Hq + 2 * Hkv) * D, H, g, b, dev, gen), g, b)
        self.o = QuantLinear(*random_quantized(H, Hq * D, g, b, dev, gen), g, b)
        self.gate_up = QuantLinear(*random_quantized(2 * F, H, g, b, dev, gen), g, b)
        self.down = QuantLinear(*random_quantized(H, F, g, b, dev, gen), g, b)
        self.norm1 = (1.0 + 0.1 * torch.randn(H, device=dev, generator=gen)).bfloat16()
        self.norm2 = (1.0 + 0.1 * torch.randn(H, device=dev, generator=gen)).bfloat16()
        self.q_norm = (1.0 + 0.1 * torch.randn(D, device=dev, generator=gen)).bfloat16()
        self.k_norm = (1.0 + 0.1 * torch.randn(D, device=dev, generator=gen)).bfloat16()

    @property
    def nbytes(self):
        return self.qkv.nbytes + self.o.nbytes + self.gate_up.nbytes + self.down.nbytes


class Qwen3Decoder:
    """Greedy generation for `batch` sequences with bf16 KV caches [B, Hkv, max_len, D]."""

    def __init__(self, cfg: Qwen3Config, batch: int, max_len: int, dev, seed: int = 0):
        self.cfg, self.B, self.max_len, self.dev = cfg, batch, max_len, dev
        gen = torch.Generator(device=dev).manual_seed(seed)
        g, b = cfg.group_size, cfg.bits
        self.embed = random_quantized(cfg.vocab, cfg.hidden, g, b, dev, gen)
        self.layers: List[Qwen3Layer] = [Qwen3Layer(cfg, dev, gen) for _ in range(cfg.n_layers)]
        self.final_norm = (1.0 + 0.1 * torch.randn(cfg.hidden, device=dev, generator=gen)).bfloat16()
        self.lm_head = QuantLinear(*random_quantized(cfg.vocab, cfg.hidden, g, b, dev, gen), g, b)
        Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.k_cache = [torch.zeros(batch, Hkv, max_len, D, **bf) for _ in range(cfg.n_layers)]
        self.v_cache = [torch.zeros(batch, Hkv, max_len, D, **bf) for _ in range(cfg.n_layers)]
        # decode-step buffers (graph inputs / outputs live here)
        self.ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.x = torch.empty(batch, cfg.hidden, **bf)
        self.h = torch.empty(batch, cfg.hidden, **bf)
        self.qkv_buf = torch.empty(batch, (Hq + 2 * Hkv) * D, **bf)
        self.q = torch.empty(batch, Hq, D, **bf)
        self.attn = torch.empty(batch, Hq, D, **bf)
        self.proj = torch.empty(batch, cfg.hidden, **bf)
        self.gu = torch.empty(batch, 2 * cfg.ffn, **bf)
        self.act = torch.empty(batch, cfg.ffn, **bf)
        self.logits = torch.empty(batch, cfg.vocab, **bf)
        self.ws = torch.zeros(max(fast.sdpa_workspace_bytes(batch, Hq, max_len, D), 4), dtype=torch.uint8,
                              device=dev)
        self._graph = None

    @property
    def weight_bytes(self):
        # every layer's weights, the lm_head, and the embedding rows of the step's tokens
        emb_row = sum(t[0].numel() * t.element_size() for t in self.embed)
        return sum(l.nbytes for l in self.layers) + self.lm_head.nbytes + self.B * emb_row

    # ---- prefill: the prompt [B, T] through the same linears at M = B*T ----
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Fill the caches with the prompt's keys / values, set the position to T and the
        ids to the greedy token after the prompt; returns those ids."""
        cfg = self.cfg
        B, T = prompt.shape
        if B != self.B or T >= self.max_len:
            raise ValueError("prompt shape does not fit the decoder")
        Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        x = fast.quantized_embedding(prompt.to(torch.int32).reshape(-1), *self.embed, cfg.group_size, cfg.bits,
                                     status=self.status)
        h = torch.empty_like(x)
        q = torch.empty(B * T, Hq, D, dtype=torch.bfloat16, device=self.dev)
        for i, L in enumerate(self.layers):
            fast.rms_norm(x, L.norm1, cfg.eps, out=h)
            qkv = L.qkv(h)
            for s in range(B):  # one call per sequence: its T rows at positions 0..T-1
                rs = slice(s * T, (s + 1) * T)
                fast.rope_qk_norm(qkv[rs], self.k_cache[i][s:s + 1], self.v_cache[i][s:s + 1], Hq, Hkv, 0, L.q_norm,
                                  L.k_norm, cfg.eps, cfg.rope_theta, tokens_per_seq=T, q_out=q[rs], status=self.status)
            qh = q.view(B, T, Hq, D).transpose(1, 2)
            kh = self.k_cache[i][:, :, :T]
            vh = self.v_cache[i][:, :, :T]
            a = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
            a = a.transpose(1, 2).reshape(B * T, Hq * D).contiguous()
            fast.add(x, L.o(a), out=x)
            fast.rms_norm(x, L.norm2, cfg.eps, out=h)
            gu = L.gate_up(h)
            fast.add(x, L.down(fast.silu_mul(gu)), out=x)
        last = x.view(B, T, -1)[:, -1].contiguous()
        fast.rms_norm(last, self.final_norm, cfg.eps, out=self.h)
        self.lm_head(self.h, out=self.logits)
        fast.argmax(self.logits, out=self.ids)
        self.pos.fill_(T)
        return self.ids

    # ---- one decode step, all on the device ----
    def step(self):
        cfg = self.cfg
        B = self.B
        small = B <= 4  # 1-4 rows: the GEMV kernels carry the RMSNorm / SwiGLU / residual fusions
        fast.quantized_embedding(self.ids, *self.embed, cfg.group_size, cfg.bits, out=self.x, status=self.status)
        x = self.x
        for i, L in enumerate(self.layers):
            if small:
                L.qkv.fused(x, norm_weight=L.norm1, eps=cfg.eps, out=self.qkv_buf)
            else:
                fast.rms_norm(x, L.norm1, cfg.eps, out=self.h)
                L.qkv(self.h, out=self.qkv_buf)
            fast.rope_qk_norm(self.qkv_buf, self.k_cache[i], self.v_cache[i], cfg.n_heads, cfg.n_kv_heads, self.pos,
                              L.q_norm, L.k_norm, cfg.eps, cfg.rope_theta, q_out=self.q, status=self.status)
            fast.sdpa_decode_at(self.q, self.k_cache[i], self.v_cache[i], self.pos, workspace=self.ws, out=self.attn)
            if small:
                L.o.fused(self.attn.view(B, -1), residual=x, out=x)
                L.gate_up.fused(x, norm_weight=L.norm2, eps=cfg.eps, out=self.gu)
                L.down.fused_swiglu(self.gu, residual=x, out=x)
            else:
                L.o(self.attn.view(B, -1), out=self.proj)
                fast.add(x, self.proj, out=x)
                fast.rms_norm(x, L.norm2, cfg.eps, out=self.h)
                L.gate_up(self.h, out=self.gu)
                fast.silu_mul(self.gu, out=self.act)
                L.down(self.act, out=self.proj)
                fast.add(x, self.proj, out=x)
        if small:
            self.lm_head.fused(x, norm_weight=self.final_norm, eps=cfg.eps, out=self.logits)
        else:
            fast.rms_norm(x, self.final_norm, cfg.eps, out=self.h)
            self.lm_head(self.h, out=self.logits)
        fast.argmax(self.logits, out=self.ids)
        fast.advance(self.pos, 1)
        return self.ids

    @property
    def launches_per_step(self):
        per_layer = 6 if self.B <= 4 else 10
        return self.cfg.n_layers * per_layer + (3 if self.B <= 4 else 4) + 1

    def capture(self, stream=None) -> "torch.cuda.CUDAGraph":
        """Capture one decode step (it reads and advances the device position, so replaying
        it generates the next token each time).  The capture itself runs no step: the
        position and ids are left as they were."""
        stream = stream or torch.cuda.Stream(self.dev)
        ids0, pos0 = self.ids.clone(), self.pos.clone()
        with torch.cuda.stream(stream):
            self.step()  # warm-up outside capture (loads kernels, sets attributes)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self.step()
            self.ids.copy_(ids0)
            self.pos.copy_(pos0)
        torch.cuda.synchronize()
        self._graph, self._gstream = g, stream
        return g

    def generate(self, steps: int, tokens_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Replay the captured step `steps` times; the sampled ids of every step are copied to
        host memory ([steps, B] int32, pinned) as they are produced."""
        if self._graph is None:
            raise RuntimeError("call capture() first")
        st = self._gstream
        if tokens_out is None:
            tokens_out = torch.empty(steps, self.B, dtype=torch.int32).pin_memory()
        with torch.cuda.stream(st):
            for t in range(steps):
                self._graph.replay()
                tokens_out[t].copy_(self.ids, non_blocking=True)
        return tokens_out
