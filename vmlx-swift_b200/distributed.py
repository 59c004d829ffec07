"""Tensor parallelism: group, all-reduce and sharded quantized linears.

Mirrors Libraries/MLXDistributedTP:
  Group(strict:backend:) / .rank / .size            Group.swift:15-65
  Collectives.allSum                               Collectives.swift:27-32 (identity for size 1, :20-28)
  AllToShardedLinear / ShardedToAllLinear          LinearLayers.swift:23-206
  shardLinear / ShardingPlan                       Sharding.swift:24-36, ShardingPlan.swift:55-154
The reference has no quantized TP ("not here yet", MLXDistributedTP/README.md:23-34);
QuantizedAllToShardedLinear / QuantizedShardedToAllLinear are the quantized
counterparts: column-parallel slices rows of (wq, scales, biases) per segment,
row-parallel slices K at whole groups, nothing is re-quantized.

One process per GPU.  The group is bootstrapped with torch.distributed (the
env:// rendezvous: RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT, or the
reference's MLX_RANK / MLX_WORLD_SIZE): every rank creates its P2P receive
buffer (vmlx_tp_create), the CUDA IPC handles are exchanged with
all_gather_object, and the data path (vmlx_tp_all_sum) never touches
torch.distributed again.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional

import torch

from . import _lib, fast, ops
from ._lib import VMLXError, check
from .llama import QuantLinear, shard_k, shard_rows
from .ops import _stream

IPC_HANDLE_BYTES = 64


def _env_rank_world():
    rank = int(os.environ.get("RANK", os.environ.get("MLX_RANK", "0")))
    world = int(os.environ.get("WORLD_SIZE", os.environ.get("MLX_WORLD_SIZE", "1")))
    return rank, world


class Group:
    """A tensor-parallel group of `size` ranks, one GPU each.

    strict=False falls back to a size-1 group when no distributed environment
    is set (Group.swift:21-24); strict=True raises instead."""

    def __init__(self, strict: bool = False, backend: str = "nvlink", max_bytes: int = 4 << 20,
                 exchange=None):
        rank, world = _env_rank_world()
        if world > 1 and exchange is None and not torch.distributed.is_initialized():
            if strict and "MASTER_ADDR" not in os.environ:
                raise VMLXError(_lib.VMLX_E_STATE, "distributed environment not set")
            torch.distributed.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
        if world == 1 and strict and os.environ.get("WORLD_SIZE") is None and os.environ.get("MLX_WORLD_SIZE") is None:
            raise VMLXError(_lib.VMLX_E_STATE, "strict group requested but no distributed environment")
        self.rank, self.size, self.backend = rank, world, backend
        self.max_bytes = max_bytes
        self._exchange = exchange or self._torch_exchange
        self._h = None
        if world > 1:
            self._connect()

    @staticmethod
    def _torch_exchange(blob: bytes) -> List[bytes]:
        out = [None] * torch.distributed.get_world_size()
        torch.distributed.all_gather_object(out, blob)
        return out

    def _connect(self):
        h = ctypes.c_void_p()
        check(_lib.lib().vmlx_tp_create(self.rank, self.size, self.max_bytes, ctypes.byref(h)))
        self._h = h
        buf = (ctypes.c_char * IPC_HANDLE_BYTES)()
        check(_lib.lib().vmlx_tp_ipc_handle(h, buf))
        handles = self._exchange(bytes(buf))
        if len(handles) != self.size:
            raise VMLXError(_lib.VMLX_E_STATE, "handle exchange returned the wrong count")
        allh = (ctypes.c_char * (IPC_HANDLE_BYTES * self.size)).from_buffer_copy(b"".join(handles))
        check(_lib.lib().vmlx_tp_open_peers(h, allh))

    @property
    def is_multi_rank(self) -> bool:
        return self.size > 1

    def all_sum(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sum of x over the group's ranks (in place when out is x).  Identity for size 1."""
        if self.size == 1:
            return x if out is None else out.copy_(x)
        out = x if out is None else out
        check(_lib.lib().vmlx_tp_all_sum(self._h, out.data_ptr(), x.data_ptr(), x.numel(), _stream(x)))
        return out

    def moe_combine_all_sum(self, y: torch.Tensor, scores: torch.Tensor, inverse_order: Optional[torch.Tensor],
                            residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None
                            ) -> torch.Tensor:
        """out [T, D] = [residual +] all_sum over the group of the score-weighted combine of this
        rank's partial expert outputs y [T*k, D] (one kernel per rank)."""
        T, k = scores.shape
        D = y.shape[-1]
        out = torch.empty(T, D, dtype=torch.bfloat16, device=y.device) if out is None else out
        sd = _lib.VMLX_F32 if scores.dtype == torch.float32 else _lib.VMLX_BF16
        if self._h is None:  # size-1 group: the plain combine
            r = ops.moe_combine(y, scores, inverse_order)
            return r if residual is None else fast.add(r, residual, out=out)
        check(_lib.lib().vmlx_tp_moe_combine_all_sum(
            self._h, out.data_ptr(), y.contiguous().data_ptr(),
            inverse_order.data_ptr() if inverse_order is not None else None, scores.contiguous().data_ptr(), sd,
            T, k, D, residual.data_ptr() if residual is not None else None, _stream(y)))
        return out

    def quantized_matmul_all_sum(self, x: torch.Tensor, ql: "QuantLinear", residual: Optional[torch.Tensor] = None,
                                 out: Optional[torch.Tensor] = None, swiglu: bool = False) -> torch.Tensor:
        """Row-parallel linear fused with its all-reduce (and residual add), decode sizes:
        out = residual + all_sum(x @ dequantized(ql)^T), one kernel per rank.  swiglu: x is the
        [.., 2K] gate||up shard and the GEMV input is silu(gate) * up (computed on load)."""
        x = x.contiguous()
        K = x.shape[-1] // (2 if swiglu else 1)
        M = x.numel() // x.shape[-1]
        N = ql.wq.shape[0]
        if out is None:
            out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
        fn = (_lib.lib().vmlx_tp_quantized_matmul_swiglu_all_sum if swiglu
              else _lib.lib().vmlx_tp_quantized_matmul_all_sum)
        check(fn(
            self._h, out.data_ptr(), x.data_ptr(), ql.wq.data_ptr(), ql.scales.data_ptr(), ql.biases.data_ptr(),
            ql.group_size, ql.bits, M, N, K, residual.data_ptr() if residual is not None else None, _stream(x)))
        return out

    def status(self) -> int:
        """VMLX_OK, or VMLX_E_PEER_TIMEOUT if a peer wait ran out since the last call (synchronous)."""
        if self._h is None:
            return _lib.VMLX_OK
        code = ctypes.c_int(0)
        check(_lib.lib().vmlx_tp_status(self._h, ctypes.byref(code)))
        return code.value

    def close(self):
        if self._h is not None:
            _lib.lib().vmlx_tp_destroy(self._h)
            self._h = None


class QuantizedAllToShardedLinear:
    """Column-parallel quantized linear: rank r keeps output rows
    [r*N/P, (r+1)*N/P) of every segment (LinearLayers.swift:59-105).  No collective."""

    def __init__(self, ql: QuantLinear, group: Group, segments: Optional[List[int]] = None):
        segs = segments or [ql.wq.shape[0]]
        r, p = group.rank, group.size
        self.local = QuantLinear(shard_rows(ql.wq, r, p, segs), shard_rows(ql.scales, r, p, segs),
                                 shard_rows(ql.biases, r, p, segs), ql.group_size, ql.bits)
        self.group = group

    def __call__(self, x, out=None):
        return self.local(x, out=out)


class QuantizedShardedToAllLinear:
    """Row-parallel quantized linear: rank r keeps input columns [r*K/P, (r+1)*K/P)
    at whole groups (LinearLayers.swift:161-190); forward = partial matmul, allSum,
    + bias once (:198-205)."""

    def __init__(self, ql: QuantLinear, group: Group, bias: Optional[torch.Tensor] = None):
        p = group.size
        k = ql.wq.shape[-1] * 32 // ql.bits
        if (k // p) % ql.group_size or k % p:
            raise VMLXError(_lib.VMLX_E_INVALID, f"K={k} does not split into whole groups over {p} ranks")
        r = group.rank
        self.local = QuantLinear(shard_k(ql.wq, r, p), shard_k(ql.scales, r, p), shard_k(ql.biases, r, p),
                                 ql.group_size, ql.bits)
        self.group, self.bias = group, bias

    def __call__(self, x_local, out=None, residual=None, fused: bool = True):
        """allSum(x_local @ W_local^T) [+ bias] [+ residual].  Decode sizes (<= 32 rows, no
        bias) run as one fused GEMV + all-reduce kernel per rank."""
        rows = x_local.numel() // x_local.shape[-1]
        if fused and self.bias is None and 1 <= rows <= 32:
            return self.group.quantized_matmul_all_sum(x_local, self.local, residual=residual, out=out)
        y = self.local(x_local)
        self.group.all_sum(y)
        if self.bias is not None:
            y = y + self.bias
        if residual is not None:
            y = fast.add(residual, y, out=out)
        elif out is not None:
            out.copy_(y)
            y = out
        return y


def group_split(n_groups: int, world: int, rank: int):
    """Whole quantization groups [g0, g1) of rank `rank` when n_groups do not divide evenly:
    the first n_groups % world ranks take one extra group (12 groups over 8 ranks:
    2,2,2,2,1,1,1,1).  Slicing at group boundaries keeps every shard a bit-exact slice of
    the quantized tensors (nothing is re-quantized)."""
    base, extra = divmod(n_groups, world)
    g0 = rank * base + min(rank, extra)
    return g0, g0 + base + (1 if rank < extra else 0)


class ShardedSwitchGLU:
    """SwitchGLU with the expert intermediate dimension sharded over a TP group (BASELINE
    config 4: Qwen3-30B-A3B's 128 experts, FFN 768, over TP=1/2/4/8).  Each rank keeps
    gate/up rows and down columns [g0*gs, g1*gs) of every expert (group_split, uneven when
    F/gs does not divide), runs the whole routed SwitchGLU + weighted combine on its slice
    (a partial sum of the block output) and all-reduces the [T, H] result once.

    The reference replicates experts under TP (Libraries/MLXDistributedTP/
    ShardingPlans+Qwen35.swift:14-19); sharding the intermediate is the TP layout of the
    MoE down projection as a row-parallel linear (LinearLayers.swift:161-205)."""

    def __init__(self, glu, group: Group):
        from .switch_layers import QuantizedSwitchLinear, SwitchGLU
        gp, up, dn = glu.gate_proj, glu.up_proj, glu.down_proj
        gs, bits = dn.group_size, dn.bits
        F = gp.output_dims
        if F % gs:
            raise VMLXError(_lib.VMLX_E_INVALID, f"intermediate {F} is not a whole number of {gs}-groups")
        g0, g1 = group_split(F // gs, group.size, group.rank)
        r0, r1 = g0 * gs, g1 * gs
        w0, w1 = r0 * bits // 32, r1 * bits // 32

        def rows(sl):  # column-parallel over the intermediate (output rows of gate / up)
            return QuantizedSwitchLinear(sl.weight[:, r0:r1].contiguous(), sl.scales[:, r0:r1].contiguous(),
                                         sl.biases[:, r0:r1].contiguous(), None, gs, bits, sl.mode)
        down = QuantizedSwitchLinear(dn.weight[..., w0:w1].contiguous(), dn.scales[..., g0:g1].contiguous(),
                                     dn.biases[..., g0:g1].contiguous(), None, gs, bits, dn.mode)
        self.local = SwitchGLU(rows(gp), rows(up), down)
        self.group, self.groups = group, (g0, g1)

    def combined(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor,
                 residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[residual +] sum_j SwitchGLU(x, indices)[:, j] * scores[:, j], reduced over the group:
        the weighted combine and the all-reduce run as one kernel (vmlx_tp_moe_combine_all_sum)."""
        y, inv = self.local._expert_outputs(x, indices)
        T = indices.reshape(-1, indices.shape[-1]).shape[0]
        return self.group.moe_combine_all_sum(y.reshape(-1, y.shape[-1]), scores.reshape(T, -1), inv, residual)
