"""Decoder-block support ops (MLXFast mirror) over the C ABI.

  rms_norm     MLXFast.rmsNorm (Source/MLX/MLXFast.swift:230)
  rope_qkv     RoPE (MLXFast.swift:26) + KVCacheSimple.update (Libraries/MLXLMCommon/KVCache.swift:452-470)
  sdpa_decode  MLXFast.scaledDotProductAttention for one query token (MLXFast.swift:118)
  silu_mul     compiledSwiGLU (Libraries/MLXLMCommon/SwitchLayers.swift:40-50)
  add          residual add
All tensors are bf16 CUDA tensors; work runs on the current stream.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import VMLXError, check
from .ops import _need_cuda, _stream


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(x, weight)
    x = x.contiguous()
    D = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    check(_lib.lib().vmlx_cuda_rms_norm(out.data_ptr(), x.data_ptr(), weight.data_ptr(), eps,
                                        x.numel() // D, D, _stream(x)))
    return out


def rope_qkv(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, n_heads: int,
             n_kv_heads: int, pos: int, base: float = 500000.0, scale: float = 1.0,
             q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate q, k of a fused qkv [B, (Hq+2Hkv)*D] at `pos`; append k, v to the
    caches [B, Hkv, max_len, D]; return q [B, Hq, D]."""
    _need_cuda(qkv, k_cache, v_cache)
    B = qkv.shape[0]
    D = k_cache.shape[-1]
    if q_out is None:
        q_out = torch.empty(B, n_heads, D, dtype=torch.bfloat16, device=qkv.device)
    check(_lib.lib().vmlx_cuda_rope_qkv(q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                        qkv.contiguous().data_ptr(), B, n_heads, n_kv_heads, D, pos,
                                        k_cache.shape[2], base, scale, _stream(qkv)))
    return q_out


def sdpa_workspace_bytes(batch: int, n_heads: int, kv_len: int, head_dim: int = 128) -> int:
    return int(_lib.lib().vmlx_cuda_sdpa_decode_workspace(batch, n_heads, kv_len, head_dim))


def sdpa_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: int,
                scale: Optional[float] = None, workspace: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [B, Hq, D] against caches [B, Hkv, max_len, D] (first kv_len positions)."""
    _need_cuda(q, k_cache, v_cache)
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    scale = D ** -0.5 if scale is None else scale
    need = sdpa_workspace_bytes(B, Hq, kv_len, D)
    if workspace is None:
        workspace = torch.zeros(max(need, 4), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    check(_lib.lib().vmlx_cuda_sdpa_decode(out.data_ptr(), q.contiguous().data_ptr(), k_cache.data_ptr(),
                                           v_cache.data_ptr(), B, Hq, Hkv, D, kv_len, k_cache.shape[2], scale,
                                           workspace.data_ptr(), workspace.numel(), _stream(q)))
    return out


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(gate_up)
    F2 = gate_up.shape[-1]
    rows = gate_up.numel() // F2
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], F2 // 2, dtype=torch.bfloat16, device=gate_up.device)
    check(_lib.lib().vmlx_cuda_silu_mul(out.data_ptr(), gate_up.contiguous().data_ptr(), rows, F2 // 2,
                                        _stream(gate_up)))
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(a, b)
    if a.shape != b.shape:
        raise VMLXError(_lib.VMLX_E_INVALID, "add: shapes differ")
    out = torch.empty_like(a) if out is None else out
    check(_lib.lib().vmlx_cuda_add(out.data_ptr(), a.contiguous().data_ptr(), b.contiguous().data_ptr(),
                                   a.numel(), _stream(a)))
    return out


# ---- the decode loop around the linears (one CUDA graph per token) ----

def quantized_embedding(ids: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                        group_size: int = 64, bits: int = 4, out: Optional[torch.Tensor] = None,
                        status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """QuantizedEmbedding (Source/MLXNN/Quantized.swift:229-236): rows of the dequantized
    table for int32 token ids [...] -> bf16 [..., dims]."""
    _need_cuda(ids, w, scales, biases)
    vocab = w.shape[0]
    dims = w.shape[1] * 32 // bits
    n = ids.numel()
    if out is None:
        out = torch.empty(*ids.shape, dims, dtype=torch.bfloat16, device=ids.device)
    check(_lib.lib().vmlx_cuda_quantized_embedding(
        out.data_ptr(), ids.contiguous().data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), group_size,
        bits, n, vocab, dims, status.data_ptr() if status is not None else None, _stream(ids)))
    return out


def rope_qk_norm(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, n_heads: int, n_kv_heads: int,
                 pos=0, q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None,
                 eps: float = 1e-6, base: float = 1000000.0, scale: float = 1.0, tokens_per_seq: int = 0,
                 q_out: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[per-head RMSNorm of q and k (Qwen3)] + RoPE + KV append.  ``pos`` is an int or an
    int32 CUDA tensor holding the position (read on the device)."""
    _need_cuda(qkv, k_cache, v_cache, q_norm, k_norm)
    rows = qkv.shape[0]
    D = k_cache.shape[-1]
    if q_out is None:
        q_out = torch.empty(rows, n_heads, D, dtype=torch.bfloat16, device=qkv.device)
    pos_dev = pos.data_ptr() if isinstance(pos, torch.Tensor) else None
    pos_int = 0 if isinstance(pos, torch.Tensor) else int(pos)
    check(_lib.lib().vmlx_cuda_rope_qk_norm(
        q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), qkv.contiguous().data_ptr(), rows, n_heads,
        n_kv_heads, D, pos_dev, pos_int, int(tokens_per_seq), k_cache.shape[2],
        q_norm.data_ptr() if q_norm is not None else None, k_norm.data_ptr() if k_norm is not None else None,
        eps, base, scale, status.data_ptr() if status is not None else None, _stream(qkv)))
    return q_out


def sdpa_decode_at(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor,
                   scale: Optional[float] = None, workspace: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """sdpa_decode over the first *pos + 1 cache positions, *pos read on the device."""
    _need_cuda(q, k_cache, v_cache, pos)
    B, Hq, D = q.shape
    Hkv, max_len = k_cache.shape[1], k_cache.shape[2]
    scale = D ** -0.5 if scale is None else scale
    if workspace is None:
        workspace = torch.zeros(max(sdpa_workspace_bytes(B, Hq, max_len, D), 4), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    check(_lib.lib().vmlx_cuda_sdpa_decode_at(out.data_ptr(), q.contiguous().data_ptr(), k_cache.data_ptr(),
                                              v_cache.data_ptr(), B, Hq, Hkv, D, pos.data_ptr(), max_len, scale,
                                              workspace.data_ptr(), workspace.numel(), _stream(q)))
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy sampling (ArgMaxSampler, Libraries/MLXLMCommon/Evaluate.swift:515-521): int32 [rows]."""
    _need_cuda(logits)
    V = logits.shape[-1]
    rows = logits.numel() // V
    out = torch.empty(rows, dtype=torch.int32, device=logits.device) if out is None else out
    check(_lib.lib().vmlx_cuda_argmax(out.data_ptr(), logits.contiguous().data_ptr(), rows, V, _stream(logits)))
    return out


def advance(counter: torch.Tensor, delta: int = 1) -> torch.Tensor:
    _need_cuda(counter)
    check(_lib.lib().vmlx_cuda_advance(counter.data_ptr(), delta, _stream(counter)))
    return counter
