"""Layer types of the quantized path (MLXNN mirror).

QuantizedLinear follows Source/MLXNN/Quantized.swift:263-417:
  - ``QuantizedLinear(weight, bias, scales, biases, group_size, bits, mode)``
    wraps pre-quantized tensors (the checkpoint initializer, :341-352);
  - ``QuantizedLinear.from_weight(w, bias, group_size, bits)`` quantizes a
    float weight (the ``init(weight:bias:groupSize:bits:mode:)`` path, :318-335);
  - ``shape`` reports the unpacked (out, in) dims (:272-275);
  - ``__call__`` is ``quantized_mm(x, w, scales, biases, transpose=True) (+ bias)``
    (:361-376).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops


class QuantizedLinear:
    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor], scales: torch.Tensor,
                 biases: Optional[torch.Tensor], group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        if mode not in ("affine", "mxfp4"):
            raise ops.VMLXError(2, f"mode {mode} not supported (affine, mxfp4)")
        self.weight = weight
        self.bias = bias
        self.scales = scales
        self.biases = biases
        self.group_size = group_size
        self.bits = bits
        self.mode = mode

    @classmethod
    def from_weight(cls, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                    group_size: int = 64, bits: int = 4, mode: str = "affine") -> "QuantizedLinear":
        if mode == "mxfp4":  # e2m1 codes with e8m0 scales per 32 values, no biases
            wq, s = ops.fp_quantized(weight, group_size=group_size, bits=bits, mode=mode)
            return cls(wq, bias, s, None, group_size, bits, mode)
        wq, s, b = ops.quantized(weight, group_size=group_size, bits=bits, mode=mode)
        return cls(wq, bias, s, b, group_size, bits, mode)

    @property
    def shape(self) -> Tuple[int, int]:
        return (self.weight.shape[-2], self.weight.shape[-1] * 32 // self.bits)

    @property
    def input_dims(self) -> int:
        return self.shape[1]

    @property
    def output_dims(self) -> int:
        return self.shape[0]

    def describe_extra(self) -> str:
        return (f"(inputDimensions={self.input_dims}, outputDimensions={self.output_dims}, "
                f"bias={'true' if self.bias is not None else 'false'})")

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.mode == "mxfp4":
            y = ops.fp_quantized_mm(x, self.weight, self.scales, self.group_size, self.bits, self.mode, out=out)
        else:
            y = ops.quantized_mm(x, self.weight, self.scales, self.biases, transpose=True,
                                 group_size=self.group_size, bits=self.bits, mode=self.mode, out=out)
        if self.bias is not None:  # the bias add on the device, in place (bf16(y + bias))
            cols = y.shape[-1]
            ops.check(ops._lib.lib().vmlx_cuda_bias_add(y.data_ptr(), y.data_ptr(), self.bias.contiguous().data_ptr(),
                                                        y.numel() // cols, cols, ops._stream(y)))
        return y
