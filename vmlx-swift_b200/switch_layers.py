"""MoE expert layers (MLXLMCommon/SwitchLayers.swift mirror).

  gather_sort / scatter_unsort   SwitchLayers.swift:64-83
  QuantizedSwitchLinear          SwitchLayers.swift:430-512
  SwitchGLU                      SwitchLayers.swift:91-367
    - sort when indices.size >= 64 (:296)
    - fused gate||up gather_qmm when indices.size <= 32 (:258-259, :288-291)
    - silu(gate) * up (:40-50), down projection, unsort, squeeze(-2)
"""
from __future__ import annotations

import os
from typing import Optional, Tuple

import torch

from . import fast, ops

# The reference fuses gate||up for <= 32 routed rows (SwitchLayers.swift:186-237); here one gather
# over the concatenated experts is never slower than two, so it is used at every size by default.
FUSED_GATE_UP_THRESHOLD = int(os.environ.get("BENCH_FUSED_GATE_UP_THRESHOLD", str(1 << 30)))


def gather_sort(x: torch.Tensor, indices: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sort the (token, slot) pairs by expert: returns (x rows in sorted order,
    sorted indices, inverse order).  Stable sort, as MLX's argsort."""
    m = indices.shape[-1]
    flat = indices.reshape(-1)
    order = torch.argsort(flat, stable=True)
    inv = torch.argsort(order, stable=True)
    xf = x.reshape(-1, *x.shape[-2:])  # flatten(start: 0, end: -3)
    return xf[order // m], flat[order], inv


def scatter_unsort(x: torch.Tensor, inv_order: torch.Tensor, shape=None) -> torch.Tensor:
    x = x[inv_order]
    if shape is not None:
        x = x.reshape(*shape, *x.shape[1:])
    return x


class QuantizedSwitchLinear:
    """Stack of E quantized expert linears: weight u32 [E, out, in*bits/32]."""

    def __init__(self, weight, scales, biases, bias=None, group_size=64, bits=4, mode="affine"):
        self.weight, self.scales, self.biases, self.bias = weight, scales, biases, bias
        self.group_size, self.bits, self.mode = group_size, bits, mode

    @classmethod
    def from_weight(cls, w: torch.Tensor, group_size=64, bits=4, mode="affine"):
        wq, s, b = ops.quantized(w, group_size=group_size, bits=bits, mode=mode)
        return cls(wq, s, b, None, group_size, bits, mode)

    @property
    def num_experts(self):
        return self.weight.shape[0]

    @property
    def output_dims(self):
        return self.weight.shape[1]

    @property
    def input_dims(self):
        return self.weight.shape[2] * 32 // self.bits

    def __call__(self, x, indices, sorted_indices: bool = False):
        y = ops.gather_quantized_mm(x, self.weight, self.scales, self.biases, rhs_indices=indices,
                                    transpose=True, group_size=self.group_size, bits=self.bits,
                                    mode=self.mode, sorted_indices=sorted_indices)
        if self.bias is not None:
            y = y + self.bias[indices].unsqueeze(-2)
        return y


class SwitchGLU:
    def __init__(self, gate_proj: QuantizedSwitchLinear, up_proj: QuantizedSwitchLinear,
                 down_proj: QuantizedSwitchLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self._fused = None

    def ensure_fused_gate_up(self):
        """Concatenate gate and up along the output axis once (SwitchLayers.swift:186-237)."""
        if self._fused is None:
            g, u = self.gate_proj, self.up_proj
            if (g.group_size, g.bits, g.mode) == (u.group_size, u.bits, u.mode):
                self._fused = QuantizedSwitchLinear(
                    torch.cat([g.weight, u.weight], 1), torch.cat([g.scales, u.scales], 1),
                    torch.cat([g.biases, u.biases], 1), None, g.group_size, g.bits, g.mode)
        return self._fused

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        fused = self.ensure_fused_gate_up()
        use_fused = fused is not None and indices.numel() <= FUSED_GATE_UP_THRESHOLD
        x = x.unsqueeze(-2).unsqueeze(-3)  # expandedDimensions(x, [-2, -3])
        do_sort = indices.numel() >= 64
        idx, inv = indices, None
        if do_sort:
            x, idx, inv = gather_sort(x, indices)
        if use_fused:
            comb = fused(x, idx, sorted_indices=do_sort)
            act = fast.silu_mul(comb)  # silu(gate) * up in one kernel over the gate||up rows
        else:
            up = self.up_proj(x, idx, sorted_indices=do_sort)
            gate = self.gate_proj(x, idx, sorted_indices=do_sort)
            act = fast.silu_mul(torch.cat([gate, up], -1))
        y = self.down_proj(act.contiguous(), idx, sorted_indices=do_sort)
        if do_sort:
            y = scatter_unsort(y, inv, indices.shape)
        return y.squeeze(-2)
