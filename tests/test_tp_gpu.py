"""GPU tests of the tensor-parallel all-reduce and the TP decoder.

Single-GPU: the size-1 group is an identity (Collectives.swift:20-28), and a
wait on a peer that never arrives ends with VMLX_E_PEER_TIMEOUT in the status
word (a flag nothing sets; the kernel's wait is bounded), leaving the context
usable.  Multi-GPU (skipped with fewer than 2 GPUs): one process per GPU
(spawned), the P2P all-reduce against a float64 sum, and a TP=2 decoder step
against the TP=1 step of the same weights."""
import ctypes
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_group_size1_identity(vm, cuda):
    g = vm.distributed.Group()
    assert g.size == 1 and not g.is_multi_rank
    x = torch.randn(4096, device=cuda).bfloat16()
    assert torch.equal(g.all_sum(x.clone()), x)
    lib = vm.lib()
    h = ctypes.c_void_p()
    assert lib.vmlx_tp_create(0, 1, 1 << 16, ctypes.byref(h)) == 0
    out = torch.empty_like(x)
    assert lib.vmlx_tp_all_sum(h, out.data_ptr(), x.data_ptr(), x.numel(), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, x)
    lib.vmlx_tp_destroy(h)


def test_peer_timeout_sets_status_and_context_survives(vm, cuda):
    lib = vm.lib()
    h0, h1 = ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.vmlx_tp_create(0, 2, 1 << 16, ctypes.byref(h0)) == 0
    assert lib.vmlx_tp_create(1, 2, 1 << 16, ctypes.byref(h1)) == 0
    assert lib.vmlx_tp_set_peer(h0, 1, lib.vmlx_tp_buffer(h1)) == 0
    assert lib.vmlx_tp_set_timeout_us(h0, 20000) == 0  # 20 ms
    x = torch.ones(1024, device=cuda).bfloat16()
    out = torch.zeros_like(x)
    # rank 1 never runs: rank 0's wait for its flag must give up and report
    assert lib.vmlx_tp_all_sum(h0, out.data_ptr(), x.data_ptr(), x.numel(), None) == 0
    code = ctypes.c_int(-1)
    assert lib.vmlx_tp_status(h0, ctypes.byref(code)) == 0
    assert code.value == vm._lib.VMLX_E_PEER_TIMEOUT
    assert lib.vmlx_tp_status(h0, ctypes.byref(code)) == 0 and code.value == 0  # cleared
    assert torch.count_nonzero(out) == 0  # no partial result written
    y = (x.float() * 2).sum().item()  # the context still works
    assert y == 2048.0
    lib.vmlx_tp_destroy(h0)
    lib.vmlx_tp_destroy(h1)


def test_fused_tp_linear_size1_and_timeout(vm, cuda):
    """world 1: the fused TP linear is the local fused GEMV (+ residual).  world 2 with a
    rank that never runs: every CTA's bounded wait gives up, the status reports it, y is
    left untouched and the context stays usable."""
    lib = vm.lib()
    g = torch.Generator(cuda).manual_seed(4)
    K, N, M = 2048, 1024, 3
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    wq, s, b = vm.quantized(w)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
    h = ctypes.c_void_p()
    assert lib.vmlx_tp_create(0, 1, 1 << 20, ctypes.byref(h)) == 0
    y = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    assert lib.vmlx_tp_quantized_matmul_all_sum(h, y.data_ptr(), x.data_ptr(), wq.data_ptr(), s.data_ptr(),
                                                b.data_ptr(), 64, 4, M, N, K, res.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, vm.ops.quantized_mm_fused(x, wq, s, b, residual=res))
    lib.vmlx_tp_destroy(h)
    h0, h1 = ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.vmlx_tp_create(0, 2, 1 << 20, ctypes.byref(h0)) == 0
    assert lib.vmlx_tp_create(1, 2, 1 << 20, ctypes.byref(h1)) == 0
    assert lib.vmlx_tp_set_peer(h0, 1, lib.vmlx_tp_buffer(h1)) == 0
    assert lib.vmlx_tp_set_timeout_us(h0, 20000) == 0
    y.zero_()
    assert lib.vmlx_tp_quantized_matmul_all_sum(h0, y.data_ptr(), x.data_ptr(), wq.data_ptr(), s.data_ptr(),
                                                b.data_ptr(), 64, 4, M, N, K, res.data_ptr(), None) == 0
    code = ctypes.c_int(-1)
    assert lib.vmlx_tp_status(h0, ctypes.byref(code)) == 0
    assert code.value == vm._lib.VMLX_E_PEER_TIMEOUT
    assert torch.count_nonzero(y) == 0
    assert (x.float() * 2).sum().isfinite().item()
    lib.vmlx_tp_destroy(h0)
    lib.vmlx_tp_destroy(h1)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        sys.path.insert(0, ROOT)
        torch.cuda.set_device(rank)
        from vmlx_b200_loader import load_package
        vm = load_package()
        dev = torch.device("cuda", rank)
        grp = vm.distributed.Group(strict=True)
        ok = []
        # all-reduce against a float64 sum of every rank's input (inputs are seeded by rank)
        for n in (8, 1000, 4096, 65536):
            xs = [torch.randn(n, generator=torch.Generator().manual_seed(100 * r + n)).bfloat16() for r in range(world)]
            ref = sum(x.double() for x in xs)
            out = grp.all_sum(xs[rank].to(dev).clone())
            err = (out.double().cpu() - ref).abs().max().item()
            ok.append(err <= 1e-2 * ref.abs().max().item() + 1e-2)
        # repeated calls (epochs / parities) inside a captured graph
        x = torch.full((4096,), float(rank + 1), device=dev).bfloat16()
        st = torch.cuda.Stream(dev)
        with torch.cuda.stream(st):
            buf = x.clone()
            grp.all_sum(buf)
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                grp.all_sum(buf)
            for _ in range(5):
                buf.copy_(x)
                g.replay()
        torch.cuda.synchronize()
        ok.append(bool(torch.all(buf.float() == world * (world + 1) / 2).item()))
        # TP=world decoder step vs TP=1 on the same weights
        cfg = vm.llama.LlamaConfig(hidden=512, n_heads=8, n_kv_heads=2, head_dim=128, ffn=1024, n_layers=2)
        x0 = torch.randn(2, cfg.hidden, generator=torch.Generator().manual_seed(7)).bfloat16().to(dev)
        full = vm.llama.LlamaDecoder(cfg, 2, max_len=48, dev=dev, seed=3, cache_fill=32)
        tp = vm.llama.LlamaDecoder(cfg, 2, max_len=48, dev=dev, seed=3, rank=rank, world=world,
                                   all_sum=grp.all_sum, cache_fill=32)
        # the TP rank's cache holds its own kv heads of the same random cache
        hk = cfg.n_kv_heads // world
        for i in range(cfg.n_layers):
            tp.k_cache[i].copy_(full.k_cache[i][:, rank * hk:(rank + 1) * hk])
            tp.v_cache[i].copy_(full.v_cache[i][:, rank * hk:(rank + 1) * hk])
        y1 = full.step(x0.clone(), 32).float()
        caches = [(k.clone(), v.clone()) for k, v in zip(tp.k_cache, tp.v_cache)]
        yp = tp.step(x0.clone(), 32).float()
        rel = ((yp - y1).abs().max() / y1.abs().max()).item()
        ok.append(rel <= 2e-2)
        # the same TP step with o_proj / down_proj as fused GEMV + all-reduce + residual kernels
        tpf = vm.llama.LlamaDecoder(cfg, 2, max_len=48, dev=dev, seed=3, rank=rank, world=world, group=grp,
                                    cache_fill=32)
        for i in range(cfg.n_layers):
            tpf.k_cache[i].copy_(caches[i][0])
            tpf.v_cache[i].copy_(caches[i][1])
        ypf = tpf.step(x0.clone(), 32).float()
        # the fused partials come from the 1-32-row GEMV's TP instance, the separate ones from the
        # kernel the shape selects: equal within the GEMV tolerance
        ok.append(((ypf - yp).abs().max() / yp.abs().max()).item() <= 2e-2)
        # fused row-parallel linear == partial GEMV -> all_sum -> add, bitwise, over graph replays
        K, N = 1024, 512
        wfull = (torch.randn(N, K, generator=torch.Generator().manual_seed(11)) * 0.02).bfloat16().to(dev)
        ql = vm.llama.QuantLinear(*vm.quantized(wfull), 64, 4)
        row = vm.distributed.QuantizedShardedToAllLinear(ql, grp)
        for M in (1, 4, 9, 32):
            xf = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).bfloat16().to(dev)
            xl = xf[:, rank * K // world:(rank + 1) * K // world].contiguous()
            res = torch.randn(M, N, generator=torch.Generator().manual_seed(50 + M)).bfloat16().to(dev)
            fused = row(xl, residual=res).float()
            sep = row(xl, residual=res, fused=False).float()
            ok.append(((fused - sep).abs().max() / sep.abs().max()).item() <= 2e-2)
        st2 = torch.cuda.Stream(dev)
        xl = torch.randn(4, K // world, generator=torch.Generator().manual_seed(rank)).bfloat16().to(dev)
        with torch.cuda.stream(st2):
            outb = torch.empty(4, N, dtype=torch.bfloat16, device=dev)
            row(xl, out=outb)
            st2.synchronize()
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=st2):
                row(xl, out=outb)
                row(xl, residual=outb, out=outb)
            for _ in range(4):
                g2.replay()
        torch.cuda.synchronize()
        once = row(xl)
        ok.append(torch.equal(outb, vm.fast.add(once, once)))
        # MoE (config 4 layout, reduced): experts' intermediate sharded over the group, the block's
        # partial outputs all-reduced, against the unsharded SwitchGLU + combine on this GPU
        E, D, F = 8, 512, 768
        gen = torch.Generator().manual_seed(21)
        mk = lambda n, kk: vm.switch_layers.QuantizedSwitchLinear.from_weight(  # noqa: E731
            (torch.randn(E, n, kk, generator=gen) * 0.02).bfloat16().to(dev))
        glu = vm.SwitchGLU(mk(F, D), mk(F, D), mk(D, F))
        xm = torch.randn(5, D, generator=gen).bfloat16().to(dev)
        lg = torch.randn(5, E, generator=gen).to(dev)
        inds, scores = vm.ops.moe_route(lg, 2)
        full_m = glu.combined(xm, inds, scores).float()
        part_m = vm.distributed.ShardedSwitchGLU(glu, grp).combined(xm, inds, scores).float()
        ok.append(((part_m - full_m).abs().max() / full_m.abs().max()).item() <= 2e-2)
        ok.append(grp.status() == 0)
        q.put((rank, ok, rel))
        grp.close()
        torch.distributed.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_all_sum_and_decoder():
    import torch.multiprocessing as mp
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, rel in res:
        assert isinstance(ok, list) and all(ok), (rank, [i for i, v in enumerate(ok) if not v] if isinstance(ok, list)
                                                  else ok, rel)
