"""CPU oracle for the quantized-linear path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker / timed baseline.  The product library
never calls it.

Wraps oracle/libvmlxq_ref.so (the C restatement in vmlxq_ref.c of the MLX
affine quantize / dequantize / qmv arithmetic, Source/Cmlx/mlx-generated/
metal/quantized.h) and adds numpy restatements of the layer logic:
  gather_sort / scatter_unsort / SwitchGLU  Libraries/MLXLMCommon/SwitchLayers.swift:64-83, 261-366
  MoE routing                               Libraries/MLXLLM/Models/Qwen3MoE.swift:137-152
  TP column/row sharding + allSum           Libraries/MLXDistributedTP/LinearLayers.swift:59-205
Seeded inputs come from numpy's PCG64 generator (np.random.default_rng(seed)).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libvmlxq_ref.so")
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        h = ctypes.CDLL(LIB)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        h.vq_quantize_f32.argtypes = [P, I64, I64, I, I, P, P, P]
        h.vq_quantize_bf16.argtypes = [P, I64, I64, I, I, P, P, P]
        h.vq_dequantize.argtypes = [P, P, P, I, I64, I64, I, I, P]
        h.vq_qmm_f64.argtypes = [P, I64, I64, P, P, P, I64, I, I, P]
        h.vq_qmm_fp32.argtypes = [P, I64, I64, P, P, P, I64, I, I, P]
        h.vq_gather_qmm_f64.argtypes = [P, I64, I64, P, P, P, I64, I64, P, P, I64, I, I, P]
        h.vq_num_threads.restype = I
        _lib = h
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- bf16 helpers (bit patterns in uint16) ----------------------------------

def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(a))


# ---- quantize / dequantize / matmul -----------------------------------------

def quantize(w, group_size=64, bits=4, dtype="bf16"):
    """Returns (wq uint32 [rows, K*bits/32], scales, biases) with scales/biases as
    bf16 bit patterns (dtype='bf16'; w given as uint16 bit patterns or floats that
    are first rounded to bf16) or float32 (dtype='f32')."""
    w = np.asarray(w)
    shape = w.shape
    K = shape[-1]
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    wq = np.zeros((rows, K * bits // 32), np.uint32)
    ng = K // group_size
    if dtype == "bf16":
        wb = w if w.dtype == np.uint16 else f32_to_bf16(w)
        wb = np.ascontiguousarray(wb.reshape(rows, K))
        s = np.zeros((rows, ng), np.uint16)
        b = np.zeros((rows, ng), np.uint16)
        rc = lib().vq_quantize_bf16(_p(wb), rows, K, group_size, bits, _p(wq), _p(s), _p(b))
    else:
        wf = np.ascontiguousarray(w.reshape(rows, K), dtype=np.float32)
        s = np.zeros((rows, ng), np.float32)
        b = np.zeros((rows, ng), np.float32)
        rc = lib().vq_quantize_f32(_p(wf), rows, K, group_size, bits, _p(wq), _p(s), _p(b))
    if rc:
        raise ValueError(f"oracle quantize failed rc={rc}")
    lead = shape[:-1]
    return wq.reshape(*lead, -1), s.reshape(*lead, ng), b.reshape(*lead, ng)


def dequantize(wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """Exact fp32 dequantization float(s)*q + float(b)."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    K = wq.shape[-1] * 32 // bits
    rows = wq.size // wq.shape[-1]
    is_bf16 = scales.dtype == np.uint16
    s = np.ascontiguousarray(scales)
    b = np.ascontiguousarray(biases)
    out = np.zeros((rows, K), np.float32)
    rc = lib().vq_dequantize(_p(wq), _p(s), _p(b), int(is_bf16), rows, K, group_size, bits, _p(out))
    if rc:
        raise ValueError("oracle dequantize failed")
    return out.reshape(*wq.shape[:-1], K)


def dequantize_bf16(wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """bf16 dequantization from bf16 scales, as affine_dequantize computes it with
    T = bfloat (quantized.h:2498-2560): bf16(bf16(s * q) + b), each operation rounded
    to nearest even.  Returns bf16 bit patterns."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    K = wq.shape[-1] * 32 // bits
    q = np.zeros(wq.shape[:-1] + (K,), np.float32)
    per = 32 // bits
    for j in range(per):
        q[..., j::per] = ((wq >> (bits * j)) & ((1 << bits) - 1)).astype(np.float32)
    s = np.repeat(bf16_to_f32(scales), group_size, axis=-1).reshape(q.shape)
    b = np.repeat(bf16_to_f32(biases), group_size, axis=-1).reshape(q.shape)
    return f32_to_bf16(round_bf16(s * q) + b)


def qmm_f64(x_bf16, wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """fp64-accumulated y = x @ deq(W)^T; x given as bf16 bit patterns [M, K]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.zeros((M, N), np.float64)
    rc = lib().vq_qmm_f64(_p(x), M, K, _p(np.ascontiguousarray(wq, np.uint32)),
                          _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                          N, group_size, bits, _p(y))
    if rc:
        raise ValueError("oracle qmm failed")
    return y


def qmm_bf16w_f64(x_bf16, wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """The tiled qmm's semantics (M > 32): W dequantized to the activation dtype
    first -- QuantizedBlockLoader writes dequantize<T>() results, T = bfloat16,
    to threadgroup memory (Source/Cmlx/mlx-generated/metal/quantized.h:525-560,
    :670-720) -- then a matmul with wide accumulation (fp64 here).  Each weight
    is rounded once to bf16 from the exact s*q + b."""
    w = round_bf16(dequantize(wq, scales, biases, group_size, bits)).astype(np.float64)
    x = bf16_to_f32(np.ascontiguousarray(x_bf16, dtype=np.uint16)).astype(np.float64)
    return x @ w.T


def qmm_fp32_bf16(x_bf16, wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """MLX-factorised fp32 GEMV (OpenMP), bf16 bit-pattern output [M, N]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.zeros((M, N), np.uint16)
    rc = lib().vq_qmm_fp32(_p(x), M, K, _p(np.ascontiguousarray(wq, np.uint32)),
                           _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                           N, group_size, bits, _p(y))
    if rc:
        raise ValueError("oracle qmm_fp32 failed")
    return y


def gather_qmm_f64(x_bf16, wq, scales, biases, lhs, rhs, group_size=64, bits=4, bf16w=False) -> np.ndarray:
    """y[b] = x[lhs[b]] @ deq(W[rhs[b]])^T in fp64 (quantized.h:1438-1491 semantics).

    x [xb, M, K] bf16 bits; W [E, N, K/pf].  lhs None: batch b reads x batch
    b*xb/nb.  Each routed expert is dequantized once (C oracle, exact fp32) and
    all batch elements routed to it are multiplied in one fp64 matmul.  bf16w: the
    tiled kernels' semantics (affine_gather_qmm_rhs, quantized.h:2197-2391, like
    qmm_bf16w_f64): each weight rounded once to bf16 first."""
    x = bf16_to_f32(np.ascontiguousarray(x_bf16, dtype=np.uint16)).astype(np.float64)
    xb, M, K = x.shape
    E, N = wq.shape[0], wq.shape[1]
    rhs = np.asarray(rhs, dtype=np.int64).reshape(-1)
    nb = rhs.size
    lhs_a = (np.arange(nb) * xb // max(nb, 1)) if lhs is None else np.asarray(lhs, np.int64).reshape(-1)
    y = np.zeros((nb, M, N), np.float64)
    for e in np.unique(rhs):
        if e < 0 or e >= E:
            continue
        sel = np.nonzero(rhs == e)[0]
        w = dequantize(wq[e], scales[e], biases[e], group_size, bits)
        w = (round_bf16(w) if bf16w else w).astype(np.float64)
        y[sel] = np.einsum("bmk,nk->bmn", x[lhs_a[sel]], w)
    return y


def num_threads() -> int:
    return lib().vq_num_threads()


# ---- layer logic (numpy) -----------------------------------------------------

def gather_sort(indices: np.ndarray):
    """Order / sorted indices / inverse order of SwitchLayers.swift:64-75 (stable)."""
    flat = indices.reshape(-1)
    order = np.argsort(flat, kind="stable")
    inv = np.argsort(order, kind="stable")
    return order, flat[order], inv


def silu(x):
    return x / (1.0 + np.exp(-x))


def switch_glu(x_bf16, gate, up, down, indices, group_size=64, bits=4, bf16w=None) -> np.ndarray:
    """Reference SwitchGLU forward: x [T, D] bf16 bits, indices [T, k];
    gate/up/down = (wq, scales, biases) stacks.  Returns float64 [T, k, D].
    Intermediate activations are rounded to bf16 where the reference holds
    bf16 arrays (gate/up outputs, silu(g)*u).  bf16w (default: T*k >= 64, the
    sorted path, and >= 8 rows per expert) selects the tiled kernels' bf16 weights."""
    T, D = x_bf16.shape
    k = indices.shape[1]
    rhs = indices.reshape(-1).astype(np.uint32)
    xb = x_bf16.reshape(T, 1, D)
    lhs = np.repeat(np.arange(T), k).astype(np.uint32)
    if bf16w is None:
        bf16w = T * k >= 64 and T * k >= 8 * gate[0].shape[0]
    g = round_bf16(gather_qmm_f64(xb, *gate, lhs, rhs, group_size, bits, bf16w).astype(np.float32))
    u = round_bf16(gather_qmm_f64(xb, *up, lhs, rhs, group_size, bits, bf16w).astype(np.float32))
    act = f32_to_bf16(round_bf16(silu(g.astype(np.float64)).astype(np.float32)) * u)
    y = gather_qmm_f64(act.reshape(T * k, 1, -1), *down, None, rhs, group_size, bits, bf16w)
    return y.reshape(T, k, -1)


def moe_route(logits: np.ndarray, k: int, norm_topk_prob: bool = False):
    """softmax(precise) -> top-k expert ids (as a sorted set per token) and scores
    (Qwen3MoE.swift:137-152).  The reference's order inside the top-k is
    implementation-defined, so ids are returned sorted ascending."""
    z = logits.astype(np.float64)
    z = np.exp(z - z.max(-1, keepdims=True))
    p = z / z.sum(-1, keepdims=True)
    top = np.argsort(-p, axis=-1, kind="stable")[:, :k]
    top = np.sort(top, axis=-1)
    sc = np.take_along_axis(p, top, -1)
    if norm_topk_prob:
        sc = sc / sc.sum(-1, keepdims=True)
    return top.astype(np.uint32), sc


# ---- decoder-block references (numpy, fp64 math with the reference's bf16 rounding points) ----

def rms_norm_ref(x_bf16, w_bf16, eps):
    """MLXFast.rmsNorm: w * bf16(x * rsqrt(mean(x^2) + eps)) -> bf16 floats."""
    x = bf16_to_f32(x_bf16).astype(np.float64)
    w = bf16_to_f32(w_bf16).astype(np.float64)
    inv = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    n = round_bf16((x * inv).astype(np.float32)).astype(np.float64)
    return round_bf16((w * n).astype(np.float32))


def rope_ref(x, pos, base, scale=1.0):
    """Non-traditional RoPE of x [..., D] (float) at position pos."""
    D = x.shape[-1]
    half = D // 2
    d = np.arange(half, dtype=np.float64)
    inv_freq = base ** (-d / half)
    th = scale * pos * inv_freq
    c, s = np.cos(th), np.sin(th)
    x1, x2 = x[..., :half].astype(np.float64), x[..., half:].astype(np.float64)
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], -1)


def sdpa_ref(q, k, v, scale):
    """q [B, Hq, D]; k, v [B, Hkv, L, D] (floats) -> [B, Hq, D] fp64 (GQA)."""
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D))
    for b in range(B):
        for h in range(Hq):
            kk, vv = k[b, h // G].astype(np.float64), v[b, h // G].astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * scale
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ vv
    return out


# ---- the reference's own kernels, compiled for the CPU (oracle/_ref) ----------------
# oracle/Makefile `make ref REF_ROOT=<reference checkout>` cuts affine_quantize,
# affine_dequantize and qmv_fast_impl out of the reference's quantized.h unchanged and
# compiles them against oracle/ref_shim.h.  These wrappers pin the C restatement above
# to them.  The library exists only where the reference checkout was available at build
# time (it then travels with the repository's built files).

REF_LIB = os.path.join(HERE, "_ref", "libmlx_metal_ref.so")
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib():
    global _ref
    if _ref is None:
        h = ctypes.CDLL(REF_LIB)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        h.ref_quantize.argtypes = [P, I, I64, I64, I, I, P, P, P]
        h.ref_dequantize.argtypes = [P, P, P, I, I64, I64, I, I, P]
        h.ref_qmv_fast.argtypes = [P, I64, I64, P, P, P, I64, I, I, P]
        _ref = h
    return _ref


def ref_quantize(w, group_size=64, bits=4, dtype="bf16"):
    """The reference's affine_quantize: same return convention as quantize()."""
    w = np.asarray(w)
    rows, K = w.shape
    wq = np.zeros((rows, K * bits // 32), np.uint32)
    ng = K // group_size
    if dtype == "bf16":
        wb = np.ascontiguousarray(w if w.dtype == np.uint16 else f32_to_bf16(w))
        s = np.zeros((rows, ng), np.uint16)
        b = np.zeros((rows, ng), np.uint16)
        rc = ref_lib().ref_quantize(_p(wb), 1, rows, K, group_size, bits, _p(wq), _p(s), _p(b))
    else:
        wf = np.ascontiguousarray(w, dtype=np.float32)
        s = np.zeros((rows, ng), np.float32)
        b = np.zeros((rows, ng), np.float32)
        rc = ref_lib().ref_quantize(_p(wf), 0, rows, K, group_size, bits, _p(wq), _p(s), _p(b))
    if rc:
        raise ValueError(f"reference quantize failed rc={rc}")
    return wq, s, b


def ref_dequantize(wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """The reference's affine_dequantize; returns the output in the scales' dtype
    (bf16 bit patterns as uint16, or float32)."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    rows = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    is_bf16 = scales.dtype == np.uint16
    out = np.zeros((rows, K), np.uint16 if is_bf16 else np.float32)
    rc = ref_lib().ref_dequantize(_p(wq), _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                                  int(is_bf16), rows, K, group_size, bits, _p(out))
    if rc:
        raise ValueError("reference dequantize failed")
    return out


def ref_qmv_fast(x_bf16, wq, scales, biases, group_size=64, bits=4) -> np.ndarray:
    """The reference's qmv_fast_impl: y bf16 bit patterns [M, N]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.zeros((M, N), np.uint16)
    rc = ref_lib().ref_qmv_fast(_p(x), M, K, _p(np.ascontiguousarray(wq, dtype=np.uint32)),
                                _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)), N,
                                group_size, bits, _p(y))
    if rc:
        raise ValueError("reference qmv_fast failed (shape not covered)")
    return y


# ---- MXFP4 (test infrastructure: restates fp_quantize / fp_dequantize / the fp qdot of
# Source/Cmlx/mlx-generated/metal/fp_quantized.h:81-100, 1749-1821 with fp4.h (e2m1) and
# fp8.h:51-80 (e8m0)) ----

_E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def _e2m1_code(x: np.ndarray) -> np.ndarray:
    """fp4_e2m1(float): the reference's threshold table (fp4.h:4-31), sign in bit 3."""
    a = np.abs(x)
    b = np.select([a > 5.0, a >= 3.5, a > 2.5, a >= 1.75, a > 1.25, a >= 0.75, a > 0.25],
                  [7, 6, 5, 4, 3, 2, 1], 0).astype(np.uint32)
    b = np.where(np.signbit(x), b | 8, b)
    return np.where(np.isnan(x), 7, b).astype(np.uint32)


def _e8m0(scale: np.ndarray):
    """fp8_e8m0(float) -> (bits, value): log2 rounded half away from zero, clamped to [-127, 127];
    bits 0 decodes to 2^-127 (fp8.h:51-80)."""
    with np.errstate(divide="ignore"):
        le = np.log2(scale.astype(np.float64))
    n = np.where(scale > 0, np.sign(le) * np.floor(np.abs(le) + 0.5), -127)
    n = np.clip(n, -127, 127).astype(np.int64)
    bits = (n + 127).astype(np.uint32)
    val = np.where(bits == 0, np.uint32(0x400000), bits << np.uint32(23)).astype(np.uint32).view(np.float32)
    return bits.astype(np.uint8), val


def mxfp4_quantize(w32: np.ndarray):
    """float32 w [rows, cols] (bf16 inputs converted exactly) -> (u32 codes [rows, cols/8], u8 scales)."""
    rows, cols = w32.shape
    g = w32.reshape(rows, cols // 32, 32).astype(np.float32)
    scale = (np.abs(g).max(-1) / np.float32(6.0)).astype(np.float32)
    sbits, sval = _e8m0(scale)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(scale[..., None] == 0, np.float32(0), (g / sval[..., None]).astype(np.float32))
    codes = _e2m1_code(q).reshape(rows, cols // 8, 8)
    words = np.zeros((rows, cols // 8), np.uint32)
    for i in range(8):
        words |= codes[..., i] << np.uint32(4 * i)
    return words, sbits


def mxfp4_values(wq: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Exact float32 values scale * e2m1 of every code: [rows, cols]."""
    rows = wq.shape[0]
    codes = np.stack([(wq >> np.uint32(4 * i)) & np.uint32(0xF) for i in range(8)], -1).reshape(rows, -1)
    v = _E2M1[codes & 7] * np.where(codes & 8, -1.0, 1.0).astype(np.float32)
    s = np.where(scales == 0, np.uint32(0x400000), scales.astype(np.uint32) << np.uint32(23)).astype(
        np.uint32).view(np.float32)
    return (v.reshape(rows, -1, 32) * s[..., None]).reshape(rows, -1).astype(np.float32)


def mxfp4_qmm_f64(x_bf16, wq, scales) -> np.ndarray:
    """x [M, K] (bf16 bits) @ (mxfp4 values)^T in float64."""
    return bf16_to_f32(x_bf16).astype(np.float64) @ mxfp4_values(wq, scales).astype(np.float64).T
