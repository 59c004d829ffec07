"""MoE expert layers (MLXLMCommon/SwitchLayers.swift mirror).

  gather_sort / scatter_unsort   SwitchLayers.swift:64-83 (device sort kernel; x rows by index)
  Qwen3MoESparseMoeBlock         Qwen3MoE.swift:116-153 (device routing and weighted sum)
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


def gather_sort(x: torch.Tensor, indices: torch.Tensor, n_experts: int):
    """gatherSort on the device (SwitchLayers.swift:64-75): a stable sort of the
    (token, slot) pairs by expert.  Returns (x flattened to [rows, 1, D], sorted expert
    ids, the x row of each sorted pair, inverse order).  The reference gathers
    x[order / k] into a copy; here the row list goes to gather_qmm as lhs_indices."""
    sorted_ids, lhs, inv = ops.moe_sort(indices, n_experts)
    return x.reshape(-1, *x.shape[-2:]), sorted_ids, lhs, inv


def scatter_unsort(x: torch.Tensor, inv_order: torch.Tensor, shape=None) -> torch.Tensor:
    """x[inv_order] (SwitchLayers.swift:77-83) with the combine kernel at weight 1 (exact)."""
    rows = inv_order.numel()
    ones = torch.ones(rows, 1, dtype=torch.float32, device=x.device)
    y = ops.moe_combine(x.reshape(rows, -1), ones, inv_order).reshape(rows, *x.shape[1:])
    if shape is not None:
        y = y.reshape(*shape, *y.shape[1:])
    return y


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

    def _workspace(self, rows: int, k: int, dev):
        """Workspace of the tensor-core sorted gather, kept and grown per layer."""
        need = ops.gather_qmm_workspace_size(rows, 1, k, self.num_experts)
        ws = getattr(self, "_ws", None)
        if ws is None or ws.numel() < need or ws.device != dev:
            ws = torch.empty(need, dtype=torch.uint8, device=dev)
            self._ws = ws
        return ws

    def __call__(self, x, indices, sorted_indices: bool = False, lhs: Optional[torch.Tensor] = None):
        ws = self._workspace(indices.numel(), x.shape[-1], x.device) if sorted_indices else None
        y = ops.gather_quantized_mm(x, self.weight, self.scales, self.biases, lhs_indices=lhs, rhs_indices=indices,
                                    transpose=True, group_size=self.group_size, bits=self.bits,
                                    mode=self.mode, sorted_indices=sorted_indices, workspace=ws)
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

    def _expert_outputs(self, x: torch.Tensor, indices: torch.Tensor):
        """Per-pair down outputs, in sorted order when the pairs were sorted.
        Returns (y [pairs, 1, D], inverse order or None)."""
        fused = self.ensure_fused_gate_up()
        use_fused = fused is not None and indices.numel() <= FUSED_GATE_UP_THRESHOLD
        x = x.unsqueeze(-2).unsqueeze(-3)  # expandedDimensions(x, [-2, -3])
        do_sort = indices.numel() >= 64
        idx, inv, lhs = indices, None, None
        if do_sort:
            x, idx, lhs, inv = gather_sort(x, indices, self.down_proj.num_experts)
        if use_fused:
            comb = fused(x, idx, sorted_indices=do_sort, lhs=lhs)
            act = fast.silu_mul(comb)  # silu(gate) * up in one kernel over the gate||up rows
        else:
            up = self.up_proj(x, idx, sorted_indices=do_sort, lhs=lhs)
            gate = self.gate_proj(x, idx, sorted_indices=do_sort, lhs=lhs)
            act = fast.silu_mul(torch.cat([gate, up], -1))
        y = self.down_proj(act.contiguous(), idx, sorted_indices=do_sort)
        return y, inv

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        y, inv = self._expert_outputs(x, indices)
        if inv is not None:
            y = scatter_unsort(y, inv, indices.shape)
        else:
            y = y.reshape(*indices.shape, *y.shape[-2:])
        return y.squeeze(-2)

    def combined(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        """sum_j SwitchGLU(x, indices)[:, j] * scores[:, j] with the unsort folded into the
        weighted sum (one kernel): the MoE block's output (Qwen3MoE.swift:150-151)."""
        y, inv = self._expert_outputs(x, indices)
        T = indices.reshape(-1, indices.shape[-1]).shape[0]
        return ops.moe_combine(y.reshape(-1, y.shape[-1]), scores.reshape(T, -1), inv)


class Qwen3MoESparseMoeBlock:
    """Qwen3MoESparseMoeBlock (Libraries/MLXLLM/Models/Qwen3MoE.swift:116-153): router
    gate, top-k routing, SwitchGLU, score-weighted sum -- every step a device kernel."""

    def __init__(self, gate, switch_mlp: SwitchGLU, top_k: int, norm_topk_prob: bool = False):
        self.gate, self.switch_mlp, self.top_k, self.norm_topk_prob = gate, switch_mlp, top_k, norm_topk_prob

    def route(self, logits: torch.Tensor):
        return ops.moe_route(logits, self.top_k, self.norm_topk_prob)

    def __call__(self, x: torch.Tensor, logits: Optional[torch.Tensor] = None) -> torch.Tensor:
        if logits is None:
            logits = self.gate(x)
        inds, scores = self.route(logits)
        return self.switch_mlp.combined(x, inds, scores)
