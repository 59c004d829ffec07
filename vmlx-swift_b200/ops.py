"""Array ops of the quantized path, mirroring MLX's Swift/C API.

Names, argument meaning and defaults follow the reference:
  quantized          Source/MLX/Ops.swift:2368-2388   (mlx_quantize)
  dequantized        Source/MLX/Ops.swift:1146-1164   (mlx_dequantize)
  quantized_mm       Source/MLX/Ops.swift:2427-2448   (mlx_quantized_matmul)
  gather_quantized_mm Source/MLX/Ops.swift:1483-1505  (mlx_gather_qmm)
Tensors are torch CUDA tensors (device memory and streams only); all compute
runs in libvmlx_cuda.so on the caller's current CUDA stream.  Errors raised
by the library surface as VMLXError, the analogue of MLX's error handler
(Source/MLX/ErrorHandler.swift:52-121).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import VMLX_BF16, VMLX_F32, VMLXError, check

__all__ = [
    "quantized", "dequantized", "quantized_mm", "gather_quantized_mm", "VMLXError",
    "pack_factor",
]


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise VMLXError(_lib.VMLX_E_INVALID, "tensors must live on a CUDA device")


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return VMLX_BF16
    if dt == torch.float32:
        return VMLX_F32
    raise VMLXError(_lib.VMLX_E_UNSUPPORTED, f"dtype {dt} not supported (bfloat16, float32)")


def pack_factor(bits: int) -> int:
    return 32 // bits


def _consecutive_broadcast(xb_shape, bshape) -> bool:
    """True when broadcasting x batches ``xb_shape`` to ``bshape`` maps flat
    batch b to x batch b*x_batches/nb: x's batch dims (right-aligned) equal
    bshape's leading dims and are 1 from the first difference on."""
    xb = (1,) * (len(bshape) - len(xb_shape)) + tuple(xb_shape)
    j = 0
    while j < len(xb) and xb[j] == bshape[j]:
        j += 1
    return all(d == 1 for d in xb[j:])


def quantized(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine"
              ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantize ``w [..., K]`` -> (wq uint32 [..., K*bits/32], scales, biases [..., K/g]).

    scales/biases take w's dtype (bf16 or f32), as MLX does.  uint32 words are
    returned as a torch.int32 tensor holding the same bits (torch has no uint32
    arithmetic; the bit pattern is what matters)."""
    _need_cuda(w)
    w = w.contiguous()
    K = w.shape[-1]
    rows = w.numel() // K if K else 0
    if K % group_size or (K * bits) % 32:
        raise VMLXError(_lib.VMLX_E_INVALID, f"last dim {K} must be a multiple of group_size {group_size}")
    wq = torch.empty(*w.shape[:-1], K * bits // 32, dtype=torch.int32, device=w.device)
    scales = torch.empty(*w.shape[:-1], K // group_size, dtype=w.dtype, device=w.device)
    biases = torch.empty_like(scales)
    check(_lib.lib().vmlx_cuda_quantize(
        wq.data_ptr(), scales.data_ptr(), biases.data_ptr(), w.data_ptr(), _dtype_code(w.dtype),
        rows, K, group_size, bits, mode.encode() if mode else None, _stream(w)))
    return wq, scales, biases


def dequantized(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
                bits: int = 4, mode: str = "affine", dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """w = scale*q + bias (fp32 math), returned in ``dtype`` (default: scales' dtype)."""
    _need_cuda(wq, scales, biases)
    dtype = dtype or scales.dtype
    K = wq.shape[-1] * 32 // bits
    rows = wq.numel() // wq.shape[-1]
    out = torch.empty(*wq.shape[:-1], K, dtype=dtype, device=wq.device)
    check(_lib.lib().vmlx_cuda_dequantize(
        out.data_ptr(), _dtype_code(dtype), wq.contiguous().data_ptr(), scales.contiguous().data_ptr(),
        biases.contiguous().data_ptr(), _dtype_code(scales.dtype), rows, K, group_size, bits,
        mode.encode() if mode else None, _stream(wq)))
    return out


def quantized_mm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: Optional[torch.Tensor],
                 transpose: bool = True, group_size: int = 64, bits: int = 4, mode: str = "affine",
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x [..., K] @ dequantized(w [N, K*bits/32])^T`` in bf16 (fp32 accumulation)."""
    _need_cuda(x, w, scales, biases)
    if x.dtype != torch.bfloat16:
        raise VMLXError(_lib.VMLX_E_UNSUPPORTED, "quantized_mm: x must be bfloat16")
    x = x.contiguous()
    K = x.shape[-1]
    N = w.shape[-2]
    M = x.numel() // K if K else 0
    if w.shape[-1] * 32 // bits != K:
        raise VMLXError(_lib.VMLX_E_INVALID, f"x K={K} does not match w K={w.shape[-1] * 32 // bits}")
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    check(_lib.lib().vmlx_cuda_quantized_matmul(
        out.data_ptr(), x.data_ptr(), w.data_ptr(), scales.data_ptr(),
        biases.data_ptr() if biases is not None else None, transpose, group_size, bits,
        mode.encode() if mode else None, M, N, K, _stream(x)))
    return out


def quantized_mm_fused(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                       group_size: int = 64, bits: int = 4, norm_weight: Optional[torch.Tensor] = None,
                       eps: float = 1e-5, residual: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode-block fusion: optional RMSNorm of x on load and residual add on store
    (M <= 32).  ``out`` may be ``residual`` for an in-place ``x += W @ norm(h)``."""
    _need_cuda(x, w, scales, biases, norm_weight, residual)
    x = x.contiguous()
    K = x.shape[-1]
    N = w.shape[-2]
    M = x.numel() // K if K else 0
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    check(_lib.lib().vmlx_cuda_quantized_matmul_fused(
        out.data_ptr(), x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), group_size, bits,
        M, N, K, norm_weight.data_ptr() if norm_weight is not None else None, eps,
        residual.data_ptr() if residual is not None else None, _stream(x)))
    return out


def quantized_mm_swiglu(gate_up: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                        group_size: int = 64, bits: int = 4, residual: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Down projection with the MLP's SwiGLU fused into the GEMV (M <= 32):
    ``[residual +] silu(gate) * up @ dequantized(w)^T`` for ``gate_up = gate | up`` [..., 2K]."""
    _need_cuda(gate_up, w, scales, biases, residual)
    gate_up = gate_up.contiguous()
    K = gate_up.shape[-1] // 2
    N = w.shape[-2]
    M = gate_up.numel() // (2 * K) if K else 0
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], N, dtype=torch.bfloat16, device=gate_up.device)
    check(_lib.lib().vmlx_cuda_quantized_matmul_swiglu(
        out.data_ptr(), gate_up.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), group_size, bits,
        M, N, K, residual.data_ptr() if residual is not None else None, _stream(gate_up)))
    return out


def gather_quantized_mm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                        biases: Optional[torch.Tensor], lhs_indices: Optional[torch.Tensor] = None,
                        rhs_indices: Optional[torch.Tensor] = None, transpose: bool = True,
                        group_size: int = 64, bits: int = 4, mode: str = "affine",
                        sorted_indices: bool = False, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MLX gather_qmm: ``y[i] = x[lhs[i]] @ dequantized(w[rhs[i]])^T`` with broadcasting.
    workspace (uint8 device tensor of gather_qmm_workspace_size bytes) lets sorted gathers with
    many rows per expert run on the tensor cores (vmlx_cuda_gather_qmm_ws).

    x [*xb, M, K]; w [E, N, K*bits/32]; indices int tensors.  The output shape
    is broadcast(index shapes, xb) + [M, N], as in MLX."""
    _need_cuda(x, w, scales, biases, lhs_indices, rhs_indices)
    if x.dtype != torch.bfloat16:
        raise VMLXError(_lib.VMLX_E_UNSUPPORTED, "gather_quantized_mm: x must be bfloat16")
    if rhs_indices is None:
        raise VMLXError(_lib.VMLX_E_INVALID, "rhs_indices is required for a stacked weight")
    x = x.contiguous()
    M, K = x.shape[-2], x.shape[-1]
    xb_shape = tuple(x.shape[:-2])
    E, N = w.shape[0], w.shape[-2]
    x_batches = 1
    for d in xb_shape:
        x_batches *= d
    if lhs_indices is None:
        bshape = torch.broadcast_shapes(xb_shape, tuple(rhs_indices.shape))
        rhs = rhs_indices.expand(bshape).reshape(-1)
        nb = rhs.numel()
        # x batch broadcast: use the implicit "consecutive" rule when it is
        # exact, else materialise lhs as the broadcast of arange(x batches).
        lhs = None if _consecutive_broadcast(xb_shape, bshape) else (
            torch.arange(x_batches, device=x.device, dtype=torch.int64)
            .reshape(xb_shape or (1,)).expand(bshape).reshape(-1))
    else:
        bshape = torch.broadcast_shapes(tuple(lhs_indices.shape), tuple(rhs_indices.shape))
        rhs = rhs_indices.expand(bshape).reshape(-1)
        lhs = lhs_indices.expand(bshape).reshape(-1)
    rhs32 = rhs.to(torch.int32).contiguous()
    lhs32 = lhs.to(torch.int32).contiguous() if lhs is not None else None
    nb = rhs32.numel()
    y = torch.empty(*bshape, M, N, dtype=torch.bfloat16, device=x.device)
    args = (y.data_ptr(), x.data_ptr(), w.data_ptr(), scales.data_ptr(),
            biases.data_ptr() if biases is not None else None,
            lhs32.data_ptr() if lhs32 is not None else None, rhs32.data_ptr(), transpose, group_size,
            bits, mode.encode() if mode else None, sorted_indices, nb, x_batches, M, N, K, E)
    if workspace is not None:
        check(_lib.lib().vmlx_cuda_gather_qmm_ws(*args, workspace.data_ptr(), workspace.numel(), _stream(x)))
    else:
        check(_lib.lib().vmlx_cuda_gather_qmm(*args, _stream(x)))
    return y


# ---- MoE routing (Libraries/MLXLLM/Models/Qwen3MoE.swift:137-152,
#      Libraries/MLXLMCommon/SwitchLayers.swift:64-83) ---------------------------------

def moe_route(logits: torch.Tensor, k: int, norm_topk_prob: bool = False):
    """softmax(logits, precise) -> (indices uint32-valued int32 [.., k], scores [.., k] in
    the logits' dtype): the k experts with the largest logits (descending), their
    softmax probabilities, optionally renormalised to sum to one."""
    _need_cuda(logits)
    lg = logits.contiguous()
    E = lg.shape[-1]
    rows = lg.numel() // E
    inds = torch.empty(*lg.shape[:-1], k, dtype=torch.int32, device=lg.device)
    scores = torch.empty(*lg.shape[:-1], k, dtype=lg.dtype, device=lg.device)
    check(_lib.lib().vmlx_cuda_moe_route(lg.data_ptr(), _dtype_code(lg.dtype), rows, E, k, norm_topk_prob,
                                         inds.data_ptr(), scores.data_ptr(), _stream(lg)))
    return inds, scores


def moe_sort(indices: torch.Tensor, n_experts: int):
    """gatherSort on the device: (sorted expert ids, token row of each sorted pair,
    inverse order), all int32 [tokens * k]; a stable sort of the flattened indices."""
    _need_cuda(indices)
    k = indices.shape[-1]
    flat = indices.reshape(-1).to(torch.int32).contiguous()
    P = flat.numel()
    sorted_ids = torch.empty(P, dtype=torch.int32, device=flat.device)
    lhs = torch.empty_like(sorted_ids)
    inv = torch.empty_like(sorted_ids)
    check(_lib.lib().vmlx_cuda_moe_sort(flat.data_ptr(), P, k, n_experts, sorted_ids.data_ptr(), lhs.data_ptr(),
                                        inv.data_ptr(), None, _stream(flat)))
    return sorted_ids, lhs, inv


def moe_combine(y: torch.Tensor, scores: torch.Tensor, inverse_order: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_j y[src(t, j)] * scores[t, j] (bf16 out); y [tokens * k, D] in sorted
    order when inverse_order is given (scatterUnsort folded in), else [tokens, k, D]."""
    _need_cuda(y, scores)
    T, k = scores.shape[0], scores.shape[-1]
    D = y.shape[-1]
    yc = y.reshape(-1, D).contiguous()
    sc = scores.reshape(T, k).contiguous()
    out = torch.empty(T, D, dtype=torch.bfloat16, device=y.device)
    inv = inverse_order.to(torch.int32).contiguous() if inverse_order is not None else None
    check(_lib.lib().vmlx_cuda_moe_combine(yc.data_ptr(), inv.data_ptr() if inv is not None else None, sc.data_ptr(),
                                           _dtype_code(sc.dtype), T, k, D, out.data_ptr(), _stream(yc)))
    return out


def gather_qmm_workspace_size(batch: int, M: int, K: int, n_experts: int) -> int:
    return int(_lib.lib().vmlx_cuda_gather_qmm_workspace_size(batch, M, K, n_experts))


# ---- MXFP4 (mode "mxfp4": e2m1 codes, one e8m0 scale per 32 values, no biases) ----

def fp_quantized(w: torch.Tensor, group_size: int = 32, bits: int = 4, mode: str = "mxfp4"):
    """w [..., K] (bf16 / f32) -> (wq int32 [..., K/8] holding u32 words, scales uint8 [..., K/32])."""
    _need_cuda(w)
    w = w.contiguous()
    K = w.shape[-1]
    rows = w.numel() // K
    wq = torch.empty(*w.shape[:-1], K // 8, dtype=torch.int32, device=w.device)
    sc = torch.empty(*w.shape[:-1], K // 32, dtype=torch.uint8, device=w.device)
    check(_lib.lib().vmlx_cuda_fp_quantize(wq.data_ptr(), sc.data_ptr(), w.data_ptr(), _dtype_code(w.dtype), rows, K,
                                           group_size, bits, mode.encode(), _stream(w)))
    return wq, sc


def fp_dequantized(wq: torch.Tensor, scales: torch.Tensor, group_size: int = 32, bits: int = 4,
                   mode: str = "mxfp4", dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    _need_cuda(wq, scales)
    K = wq.shape[-1] * 8
    rows = wq.numel() * 8 // K
    out = torch.empty(*wq.shape[:-1], K, dtype=dtype, device=wq.device)
    check(_lib.lib().vmlx_cuda_fp_dequantize(out.data_ptr(), _dtype_code(dtype), wq.data_ptr(), scales.data_ptr(), rows,
                                             K, group_size, bits, mode.encode(), _stream(wq)))
    return out


def fp_quantized_mm(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, group_size: int = 32, bits: int = 4,
                    mode: str = "mxfp4", out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(x, wq, scales)
    x = x.contiguous()
    K = x.shape[-1]
    N = wq.shape[-2]
    M = x.numel() // K
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    check(_lib.lib().vmlx_cuda_fp_quantized_matmul(out.data_ptr(), x.data_ptr(), wq.data_ptr(), scales.data_ptr(),
                                                   group_size, bits, mode.encode(), M, N, K, _stream(x)))
    return out
