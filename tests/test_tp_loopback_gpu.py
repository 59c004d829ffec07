"""The tensor-parallel collectives on ONE GPU, through the C ABI: a loopback group
(vmlx_tp_create_loopback) runs all `world` ranks of a group in one cooperative grid
on this device, with the same kernels, {value, epoch} words, slot parities and
rank-order sums as a group with one GPU per rank.  This puts the multi-rank numerics
of vmlx_tp_all_sum and vmlx_tp_quantized_matmul_(swiglu_)all_sum in front of every
single-GPU run (separate launches that wait on one another are never used: the
ranks share one launch).

Bars: all_sum is bitwise equal to the rank-order fp32 sum of the ranks' bf16 inputs
(the reduction's definition) on every rank; the fused row-parallel linear matches
residual + bf16(sum_r bf16(partial_r)) with the partials from the fp64 oracle at the
GEMV tolerance (max 1e-2 / mean 1e-3 relative), and every rank holds the same bits;
graph replays (epochs and parities advancing on the device) repeat the result."""
import ctypes

import numpy as np
import pytest
import torch

from test_quant_gpu import bits_of, check_close, u32

pytestmark = pytest.mark.gpu


def _loopback(vm, world, max_bytes=1 << 20):
    h = ctypes.c_void_p()
    rc = vm.lib().vmlx_tp_create_loopback(world, max_bytes, ctypes.byref(h))
    assert rc == 0, vm.lib().vmlx_last_error()
    return h


def _status(vm, h):
    code = ctypes.c_int(-1)
    assert vm.lib().vmlx_tp_status(h, ctypes.byref(code)) == 0
    return code.value


def _rank_order_sum(xs):
    s = torch.zeros_like(xs[0], dtype=torch.float32)
    for x in xs:
        s = s + x.float()
    return s.bfloat16()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_loopback_all_sum_bitwise(vm, cuda, world):
    lib = vm.lib()
    h = _loopback(vm, world)
    st = torch.cuda.current_stream().cuda_stream
    for n in (8, 1000, 4096, 65536):  # word protocol up to max_bytes / 8, flags above
        g = torch.Generator(device=cuda).manual_seed(1000 * world + n)
        xin = torch.randn(world, n, device=cuda, generator=g).bfloat16()
        out = torch.full_like(xin, float("nan"))
        assert lib.vmlx_tp_all_sum(h, out.data_ptr(), xin.data_ptr(), n, st) == 0, lib.vmlx_last_error()
        torch.cuda.synchronize()
        assert _status(vm, h) == 0
        ref = _rank_order_sum(list(xin))
        for r in range(world):
            assert torch.equal(out[r], ref), (n, r)
    lib.vmlx_tp_destroy(h)


def test_loopback_all_sum_graph_replay(vm, cuda):
    lib = vm.lib()
    world, n = 4, 4096
    h = _loopback(vm, world)
    x = torch.stack([torch.full((n,), float(r + 1), device=cuda) for r in range(world)]).bfloat16()
    buf = x.clone()
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        assert lib.vmlx_tp_all_sum(h, buf.data_ptr(), buf.data_ptr(), n, s.cuda_stream) == 0
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            assert lib.vmlx_tp_all_sum(h, buf.data_ptr(), buf.data_ptr(), n, s.cuda_stream) == 0
        for _ in range(5):
            buf.copy_(x)
            graph.replay()
    torch.cuda.synchronize()
    assert _status(vm, h) == 0
    assert bool(torch.all(buf.float() == world * (world + 1) / 2).item())
    lib.vmlx_tp_destroy(h)


def _shards(vm, cuda, world, N, K, gs, bits, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    wq, s, b = vm.quantized(w, group_size=gs, bits=bits)
    kr = K // world
    pw, pg = kr * bits // 32, kr // gs
    parts = [(wq[:, r * pw:(r + 1) * pw].contiguous(), s[:, r * pg:(r + 1) * pg].contiguous(),
              b[:, r * pg:(r + 1) * pg].contiguous()) for r in range(world)]
    stacked = tuple(torch.cat([p[i] for p in parts], 0).contiguous() for i in range(3))
    return parts, stacked


@pytest.mark.parametrize("world,M,N,K", [(w, m, 1024, 2048) for w in (2, 4) for m in (1, 4, 9, 32)] +
                         [(8, 1, 4096, 4096), (8, 4, 4096, 14336)])
def test_loopback_row_parallel_linear(vm, orc, cuda, world, M, N, K):
    """world 8 with the Llama o_proj / down_proj shards of TP=8 (K 512 / 1792 per rank)."""
    lib = vm.lib()
    gs, bits = 64, 4
    kr = K // world
    parts, (wst, sst, bst) = _shards(vm, cuda, world, N, K, gs, bits, 11 + M)
    g = torch.Generator(device=cuda).manual_seed(M)
    x = torch.randn(world, M, kr, device=cuda, generator=g).bfloat16()
    res = torch.randn(world, M, N, device=cuda, generator=g).bfloat16()
    res[1:] = res[0]  # every rank adds the same residual (the replicated hidden state)
    h = _loopback(vm, world)
    y = torch.full((world, M, N), float("nan"), device=cuda, dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.vmlx_tp_quantized_matmul_all_sum(h, y.data_ptr(), x.data_ptr(), wst.data_ptr(), sst.data_ptr(),
                                              bst.data_ptr(), gs, bits, M, N, kr, res.data_ptr(), st)
    assert rc == 0, lib.vmlx_last_error()
    torch.cuda.synchronize()
    assert _status(vm, h) == 0
    for r in range(1, world):
        assert torch.equal(y[r], y[0]), r  # the same bits on every rank
    part = np.zeros((M, N), np.float64)
    for r, (pq, ps, pb) in enumerate(parts):
        p = orc.qmm_f64(bits_of(x[r]), u32(pq), bits_of(ps), bits_of(pb), gs, bits)
        part += orc.round_bf16(p.astype(np.float32)).astype(np.float64)
    ref = res[0].double().cpu().numpy() + orc.round_bf16(part.astype(np.float32)).astype(np.float64)
    check_close(y[0].float().cpu().numpy(), ref)
    lib.vmlx_tp_destroy(h)


def test_loopback_row_parallel_swiglu_and_replay(vm, orc, cuda):
    """The SwiGLU-fused down projection, then graph replays of two chained fused calls
    (the second adds onto the first's output as its residual)."""
    lib = vm.lib()
    world, M, N, K, gs, bits = 2, 4, 512, 1024, 64, 4
    kr = K // world
    parts, (wst, sst, bst) = _shards(vm, cuda, world, N, K, gs, bits, 5)
    g = torch.Generator(device=cuda).manual_seed(3)
    gu = torch.randn(world, M, 2 * kr, device=cuda, generator=g).bfloat16()
    h = _loopback(vm, world)
    st = torch.cuda.current_stream().cuda_stream
    y = torch.empty(world, M, N, device=cuda, dtype=torch.bfloat16)
    rc = lib.vmlx_tp_quantized_matmul_swiglu_all_sum(h, y.data_ptr(), gu.data_ptr(), wst.data_ptr(),
                                                     sst.data_ptr(), bst.data_ptr(), gs, bits, M, N, kr, None, st)
    assert rc == 0, lib.vmlx_last_error()
    torch.cuda.synchronize()
    assert torch.equal(y[1], y[0])
    part = np.zeros((M, N), np.float64)
    for r, (pq, ps, pb) in enumerate(parts):
        xa = vm.fast.silu_mul(gu[r])
        p = orc.qmm_f64(bits_of(xa), u32(pq), bits_of(ps), bits_of(pb), gs, bits)
        part += orc.round_bf16(p.astype(np.float32)).astype(np.float64)
    check_close(y[0].float().cpu().numpy(), orc.round_bf16(part.astype(np.float32)))
    once = y.clone()
    s = torch.cuda.Stream(cuda)
    out = torch.empty_like(y)
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for resid in (None, out):
                assert lib.vmlx_tp_quantized_matmul_swiglu_all_sum(
                    h, out.data_ptr(), gu.data_ptr(), wst.data_ptr(), sst.data_ptr(), bst.data_ptr(), gs, bits, M,
                    N, kr, resid.data_ptr() if resid is not None else None, s.cuda_stream) == 0
        for _ in range(4):
            graph.replay()
    torch.cuda.synchronize()
    assert _status(vm, h) == 0
    assert torch.equal(out, vm.fast.add(once, once))
    lib.vmlx_tp_destroy(h)


def test_loopback_rejects_bad_world(vm, cuda):
    h = ctypes.c_void_p()
    assert vm.lib().vmlx_tp_create_loopback(1, 1 << 16, ctypes.byref(h)) != 0
    assert vm.lib().vmlx_tp_create_loopback(9, 1 << 16, ctypes.byref(h)) != 0


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("score_dtype", [torch.float32, torch.bfloat16])
def test_loopback_moe_combine_all_sum(vm, cuda, world, score_dtype):
    """The MoE block output under expert-intermediate TP: each rank's weighted combine of its
    partial expert outputs, all-reduced in the same kernel.  Per rank it must equal the
    separate combine kernel's output (bitwise), and the result the rank-order sum of those,
    plus the residual."""
    lib = vm.lib()
    T, k, D = 33, 8, 2048
    g = torch.Generator(device=cuda).manual_seed(world)
    y = torch.randn(world, T * k, D, device=cuda, generator=g).bfloat16()
    inv = torch.stack([torch.randperm(T * k, device=cuda, generator=g) for _ in range(world)]).to(torch.int32)
    inv[1:] = inv[0]  # routing is replicated: every rank holds the same order and scores
    sc = torch.rand(T, k, device=cuda, generator=g).to(score_dtype)
    scores = sc.expand(world, T, k).contiguous()
    res = torch.randn(T, D, device=cuda, generator=g).bfloat16().expand(world, T, D).contiguous()
    h = _loopback(vm, world, max_bytes=T * D * 8)
    out = torch.full((world, T, D), float("nan"), device=cuda, dtype=torch.bfloat16)
    sd = vm._lib.VMLX_F32 if score_dtype == torch.float32 else vm._lib.VMLX_BF16
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.vmlx_tp_moe_combine_all_sum(h, out.data_ptr(), y.data_ptr(), inv.data_ptr(), scores.data_ptr(), sd, T,
                                         k, D, res.data_ptr(), st)
    assert rc == 0, lib.vmlx_last_error()
    torch.cuda.synchronize()
    assert _status(vm, h) == 0
    parts = [vm.ops.moe_combine(y[r], sc, inv[r]) for r in range(world)]
    ref = vm.fast.add(_rank_order_sum(parts), res[0])
    for r in range(world):
        assert torch.equal(out[r], ref), r
    lib.vmlx_tp_destroy(h)
