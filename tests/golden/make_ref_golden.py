"""Generates tests/golden/ref_kernels.npz: outputs of the reference's own
affine_quantize, affine_dequantize and qmv_fast_impl (Source/Cmlx/mlx-generated/
metal/quantized.h), compiled for the CPU by `make -C oracle ref REF_ROOT=<reference
checkout>` into oracle/_ref/libmlx_metal_ref.so, on small seeded inputs.

    python tests/golden/make_ref_golden.py

The fixtures let the oracle tests pin the C restatement to the reference on machines
where the reference checkout (and so oracle/_ref) is absent.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle  # noqa: E402


def weights(rng, rows, cols, gs):
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    w[0, :gs] = -np.abs(w[0, :gs])      # all-negative group: w_max starts at 0
    w[1, :gs] = 0                       # all-zero group
    w[2, :gs] = 0.125                   # constant group
    w[3, gs:2 * gs] = np.linspace(-1, 3, gs)
    return w


def main():
    assert oracle.ref_available(), "build oracle/_ref first: make -C oracle ref REF_ROOT=<reference checkout>"
    out = {}
    for gs in (32, 64, 128):
        for bits in (2, 4, 8):
            rng = np.random.default_rng(1000 + gs * 10 + bits)
            w = weights(rng, 16, 4 * gs, gs)
            wb = oracle.f32_to_bf16(w)
            key = f"g{gs}b{bits}"
            out[f"{key}_w_bf16"] = wb
            q, s, b = oracle.ref_quantize(wb, gs, bits, "bf16")
            out[f"{key}_q"], out[f"{key}_s"], out[f"{key}_b"] = q, s, b
            out[f"{key}_deq_bf16"] = oracle.ref_dequantize(q, s, b, gs, bits)
            out[f"{key}_w_f32"] = w
            qf, sf, bf = oracle.ref_quantize(w, gs, bits, "f32")
            out[f"{key}_qf"], out[f"{key}_sf"], out[f"{key}_bf"] = qf, sf, bf
            out[f"{key}_deq_f32"] = oracle.ref_dequantize(qf, sf, bf, gs, bits)
    for bits in (4, 8):
        rng = np.random.default_rng(77 + bits)
        K, N, M = 1024, 64, 3
        wb = oracle.f32_to_bf16(rng.normal(0, 0.02, (N, K)).astype(np.float32))
        x = oracle.f32_to_bf16(rng.normal(0, 1, (M, K)).astype(np.float32))
        q, s, b = oracle.ref_quantize(wb, 64, bits, "bf16")
        out[f"qmv_b{bits}_x"], out[f"qmv_b{bits}_q"], out[f"qmv_b{bits}_s"], out[f"qmv_b{bits}_b"] = x, q, s, b
        out[f"qmv_b{bits}_y"] = oracle.ref_qmv_fast(x, q, s, b, 64, bits)
    np.savez_compressed(os.path.join(HERE, "ref_kernels.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
