"""Benchmark of the quantized-linear decode path on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|gemv] [--impl ours|reference]

Prints ONE JSON line (rank 0).  Workloads:
  gemv    BASELINE config 1: one MLX affine quantized_matmul, x [1,4096] bf16,
          W [4096,4096] 4-bit g64; a step is one call.  32 weight copies are
          rotated (302 MB > 2x L2) so every call streams its weights from HBM.
  decode  BASELINE config 3: a decode step of the 32-block Llama-3-8B-shaped decoder
          stack (4-bit g64, bf16 KV cache), TP=N over the ranks of the launch.
The reference arm (--impl reference) times the CPU restatement of the
reference arithmetic (oracle/libvmlxq_ref.so, OpenMP on all host cores).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK = 6650.0
TF_FALLBACK = 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return HBM_FALLBACK, TF_FALLBACK, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_traffic(kernel_key: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(kernel_key)
    return None


# ---------------------------------------------------------------------------
# GEMV workload (BASELINE configs 1 and 2)
# ---------------------------------------------------------------------------

def gemv_bytes(M, N, K, bits, gs):
    return N * K * bits // 8 + (N * K // gs) * 4 + 2 * M * K + 2 * M * N


def make_quantized(vm, torch, dev, N, K, bits, gs, copies, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for c in range(copies):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        out.append(vm.quantized(w, group_size=gs, bits=bits))
        del w
    return out


def time_graph_calls(torch, fn_list, reps, warmup, stream):
    """Capture the calls in fn_list into one CUDA graph; replay it; return
    seconds per call (CUDA events on the launching stream)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for f in fn_list:  # warm / JIT
            f()
        stream.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for f in fn_list:
                f()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        for _ in range(warmup):
            g.replay()
        stream.synchronize()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (reps * len(fn_list))


def bench_gemv(args, torch, vm, dev):
    hbm, tf, tf_s, peak_src = peaks()
    stream = torch.cuda.Stream(dev)
    M, N, K, bits, gs = 1, 4096, 4096, 4, 64
    copies = 32
    ws = make_quantized(vm, torch, dev, N, K, bits, gs, copies, 0)
    x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(1)).bfloat16()
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    calls = [(lambda wsb=wsb: vm.quantized_mm(x, *wsb, out=y)) for wsb in ws]
    reps = max(1, args.steps // copies)
    vm.lib().vmlx_set_launch_overlap(1)  # weights are static: let each call prefetch during the previous
    with ClockSampler(dev.index or 0) as clk:
        t_call = time_graph_calls(torch, calls, reps, max(3, args.warmup), stream)
    nbytes = gemv_bytes(M, N, K, bits, gs)
    achieved = nbytes / t_call / 1e9
    # the reference's chained method (QuantMatmulCeilingTests.swift:52-69): 12 dependent calls, each
    # call's output the next call's input (square matrix), weights rotated over the copies
    bufs = [x] + [torch.empty(M, N, device=dev, dtype=torch.bfloat16) for _ in range(12)]
    chain = [(lambda i=i: vm.quantized_mm(bufs[i], *ws[i % copies], out=bufs[i + 1])) for i in range(12)]
    t_chain = time_graph_calls(torch, chain, max(4, args.steps // 12), 3, stream)

    # end to end through the public API: pinned host x -> device, call, y -> host
    xh = torch.empty(M, K, dtype=torch.bfloat16).pin_memory()
    xh.copy_(x.cpu())
    yh = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_e2e = max(args.steps, 64)
    with torch.cuda.stream(stream):
        xd = torch.empty_like(x)
        for i in range(args.warmup):
            xd.copy_(xh, non_blocking=True)
            yd = vm.quantized_mm(xd, *ws[i % copies])
            yh.copy_(yd, non_blocking=True)
        stream.synchronize()
        e0.record(stream)
        for i in range(n_e2e):
            xd.copy_(xh, non_blocking=True)
            yd = vm.quantized_mm(xd, *ws[i % copies])
            yh.copy_(yd, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3 / n_e2e

    # config 2 sweep (HBM regime, 8 rotating copies of each matrix)
    sweep = {}
    if not args.quick:
        for (KK, NN) in [(4096, 14336), (14336, 4096)]:
            for b in (4, 8):
                wsw = make_quantized(vm, torch, dev, NN, KK, b, 64, 8, 7)
                for MM in (1, 8, 32, 128, 512):
                    xx = torch.randn(MM, KK, device=dev).bfloat16()
                    yy = torch.empty(MM, NN, device=dev, dtype=torch.bfloat16)
                    cl = [(lambda w_=w_, xx=xx, yy=yy, b=b: vm.quantized_mm(xx, *w_, bits=b, out=yy))
                          for w_ in wsw]
                    t = time_graph_calls(torch, cl, 8, 3, stream)
                    gbs = gemv_bytes(MM, NN, KK, b, 64) / t / 1e9
                    row = {"us": round(t * 1e6, 2), "GBps": round(gbs, 1), "frac_8TBps": round(gbs / 8000, 3),
                           "kernel": ("qgemv_kernel / qmv_kernel (CUDA cores)" if MM <= 4 else
                                      "qmm_tc_kernel (tcgen05, TMEM)")}
                    if MM > 4:  # tensor-core regime: the tensor roofline as well
                        tfs = 2.0 * MM * NN * KK / t / 1e12
                        row.update({"TFLOPs": round(tfs, 1), "frac_of_bf16_peak": round(tfs / tf, 4)})
                    sweep[f"K{KK}_N{NN}_b{b}_M{MM}"] = row
                del wsw
    cpu = None if args.no_cpu else cpu_baseline_gemv(M, N, K, bits, gs, seconds=args.cpu_seconds)
    if args.profile:
        # one eager instance of each profiled kernel inside an NVTX range (ncu --nvtx-include vmlx_profile/):
        # the config-1 GEMV and the config-2 M=512 gate/up GEMM on the tensor-core path
        wg = make_quantized(vm, torch, dev, 14336, 4096, 4, 64, 1, 9)[0]
        xg = torch.randn(512, 4096, device=dev).bfloat16()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("vmlx_profile")
        vm.quantized_mm(x, *ws[0], out=y)
        vm.quantized_mm(xg, *wg)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    return {
        "metric": "quantized GEMV HBM GB/s (4096x4096, 4-bit g64, M=1)",
        "value": round(achieved, 1), "unit": "GB/s", "higher_is_better": True,
        "ms_per_step": t_call * 1e3, "dtype": "bf16",
        "config": {"workload": "BASELINE config 1: MLX affine quantized_matmul GEMV", "M": M, "N": N, "K": K,
                   "bits": bits, "group_size": gs, "weight_copies_rotated": copies,
                   "l2": "inputs rotated over 302 MB of weight copies (> 2x L2)", "graph": "CUDA graph of 32 calls",
                   "launch_overlap": "on (programmatic dependent launch)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                     "frac_of_8TBps": round(achieved / 8000, 4),
                     "traffic": load_traffic("qgemv_kernel_4096x4096_b4_M1"),
                     "chained_x12": {"us_per_call": round(t_chain * 1e6, 2),
                                     "GBps": round(nbytes / t_chain / 1e9, 1),
                                     "method": "12 dependent calls in one CUDA graph (output feeds the next input)"},
                     "algorithmic_bytes_per_launch": nbytes},
        "e2e": {"value": round(nbytes / t_e2e / 1e9, 2), "unit": "GB/s", "us_per_call": round(t_e2e * 1e6, 2),
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2},
        "gpu_launches": reps * copies,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "sweep_config2": sweep,
    }


def cpu_baseline_gemv(M, N, K, bits, gs, seconds=10.0):
    """Times the CPU restatement of the reference GEMV (OpenMP, all host threads)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    rng = np.random.default_rng(0)
    wb = oracle.f32_to_bf16(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    wq, s, b = oracle.quantize(wb, gs, bits)
    xb = oracle.f32_to_bf16(rng.normal(0, 1, (M, K)).astype(np.float32))
    oracle.qmm_fp32_bf16(xb, wq, s, b, gs, bits)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.qmm_fp32_bf16(xb, wq, s, b, gs, bits)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(gemv_bytes(M, N, K, bits, gs) / dt / 1e9, 3), "unit": "GB/s",
            "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n} calls of the {N}x{K} b{bits} g{gs} M={M} GEMV over {seconds:.0f} s",
            "us_per_call": round(dt * 1e6, 1)}


# ---------------------------------------------------------------------------
# MoE workload: Qwen3-30B-A3B-shaped SwitchGLU layer
# ---------------------------------------------------------------------------

MOE_H, MOE_E, MOE_F, MOE_K = 2048, 128, 768, 8
MOE_EXPERT_BYTES = 3 * MOE_F * MOE_H // 2 + 3 * (MOE_F * MOE_H // 64) * 4  # gate+up+down, 4-bit g64


def bench_moe(args, torch, vm, dev, grp=None):
    """One MoE layer for T tokens: router softmax -> top-8 of synthetic logits ~N(0,1)
    (moe_route kernel), the expert sort when T*8 >= 64 (moe_sort), SwitchGLU over the routed
    experts (gather_qmm gate||up, SwiGLU, gather_qmm down), and the score-weighted combine
    with the unsort folded in (moe_combine) -- all inside the timed region.  Bytes = distinct experts routed x their packed weights (the
    reference's per-expert weight stream) + activations."""
    hbm, tf, tf_s, peak_src = peaks()
    T = args.tokens
    stream = torch.cuda.Stream(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    copies = 4  # rotated layers (> L2: 4 x 340 MB of experts)

    def experts(n, k):
        w = (torch.randn(MOE_E, n, k, device=dev, generator=g) * 0.02).bfloat16()
        return vm.switch_layers.QuantizedSwitchLinear.from_weight(w)
    layers = []
    for _ in range(copies):
        gate, up, down = experts(MOE_F, MOE_H), experts(MOE_F, MOE_H), experts(MOE_H, MOE_F)
        layer = vm.switch_layers.SwitchGLU(gate, up, down)
        layer.ensure_fused_gate_up()
        layers.append(layer)
    blocks = [vm.switch_layers.Qwen3MoESparseMoeBlock(None, L, MOE_K) for L in layers]
    world = grp.size if grp is not None else 1
    # TP: every expert's intermediate sharded over the group; the weighted combine and the
    # all-reduce run as one kernel per rank (ShardedSwitchGLU -> vmlx_tp_moe_combine_all_sum)
    sharded = [vm.distributed.ShardedSwitchGLU(L, grp) for L in layers] if world > 1 else None
    if sharded:
        for sL in sharded:
            if hasattr(sL.local, "ensure_fused_gate_up"):
                sL.local.ensure_fused_gate_up()
        del layers[:]
        layers.extend(range(copies))
    logits = torch.randn(T, MOE_E, device=dev, generator=g)  # router logits ~N(0,1), fp32
    inds, _ = vm.ops.moe_route(logits, MOE_K)
    x = torch.randn(T, MOE_H, device=dev, generator=g).bfloat16()
    distinct = int(torch.unique(inds).numel())

    def layer_fn(L, xin):
        # routing (softmax + top-8), sort, SwitchGLU and the weighted combine: device kernels
        if sharded:
            i, sc = vm.ops.moe_route(logits, MOE_K)
            return sharded[layers.index(L)].combined(xin, i, sc)
        return blocks[layers.index(L)](xin, logits)
    outs = [None] * copies
    calls = [(lambda i=i: outs.__setitem__(i, layer_fn(layers[i], x))) for i in range(copies)]
    with ClockSampler(dev.index or 0) as clk:
        t_layer = time_graph_calls(torch, calls, max(2, args.steps // copies), max(3, args.warmup), stream)
    if world > 1:
        tt = torch.tensor([t_layer], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_layer = tt.item()
    nbytes = distinct * MOE_EXPERT_BYTES // world + T * MOE_H * 2 * 2 + T * MOE_K * (MOE_F // world) * 2 * 3
    achieved = nbytes / t_layer / 1e9

    # end to end: pinned host tokens in, layer, host out
    xh = x.cpu().pin_memory()
    yh = torch.empty(T, MOE_H, dtype=torch.bfloat16).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_e2e = max(16, args.steps // 2)
    with torch.cuda.stream(stream):
        xd = torch.empty_like(x)
        for i in range(3):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(layer_fn(layers[i % copies], xd), non_blocking=True)
        stream.synchronize()
        e0.record(stream)
        for i in range(n_e2e):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(layer_fn(layers[i % copies], xd), non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3 / n_e2e
    cpu = None if args.no_cpu else cpu_baseline_moe(T, seconds=args.cpu_seconds)
    return {
        "metric": f"MoE SwitchGLU layer tokens/s (Qwen3-30B-A3B-shaped, top-8 of 128 experts, 4-bit g64, T={T})",
        "value": round(T / t_layer, 2), "unit": "tokens/s", "higher_is_better": True,
        "ms_per_step": t_layer * 1e3, "dtype": "bf16",
        "config": {"workload": f"BASELINE config 4: SwitchGLU gather_qmm, hidden {MOE_H}, {MOE_E} experts, expert FFN "
                               f"{MOE_F}, top-{MOE_K} routing from softmax of random logits, T={T} tokens, TP={world}",
                   "tokens": T, "parallelism": f"tp{world}", "distinct_experts": distinct, "layers_rotated": copies,
                   "l2": f"{copies} rotated layers of {MOE_E * MOE_EXPERT_BYTES / 1e6:.0f} MB of experts (> L2)",
                   "graph": "layer calls captured in a CUDA graph"},
        "roofline": {"bound": "hbm", "kernel": "gather_qmm kernels (SwitchGLU gate||up and down), per rank",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": peak_src, "algorithmic_bytes_per_layer": nbytes, "traffic": None},
        "e2e": {"value": round(T / t_e2e, 2), "unit": "tokens/s", "ms_per_step": round(t_e2e * 1e3, 3),
                "h2d_bytes_per_step": T * MOE_H * 2, "d2h_bytes_per_step": T * MOE_H * 2},
        "gpu_launches": None,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }


def cpu_baseline_moe(T, seconds=10.0):
    """The oracle's SwitchGLU (numpy per routed expert over the C dequantization) on a sample."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    rng = np.random.default_rng(0)

    def qw(n, k):
        wq, s, b = [], [], []
        for _ in range(MOE_E):
            a, c, d = oracle.quantize(oracle.f32_to_bf16(rng.normal(0, 0.02, (n, k)).astype(np.float32)), 64, 4)
            wq.append(a); s.append(c); b.append(d)
        return np.stack(wq), np.stack(s), np.stack(b)
    gate, up, down = qw(MOE_F, MOE_H), qw(MOE_F, MOE_H), qw(MOE_H, MOE_F)
    x = oracle.f32_to_bf16(rng.normal(size=(T, MOE_H)).astype(np.float32))
    idx = np.argsort(-rng.normal(size=(T, MOE_E)), -1)[:, :MOE_K]
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds or n == 0:
        oracle.switch_glu(x, gate, up, down, idx, 64, 4)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(T / dt, 3), "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n} SwitchGLU layers of {T} tokens (oracle: C dequantization + numpy matmuls per routed expert)",
            "ms_per_layer": round(dt * 1e3, 1)}


# ---------------------------------------------------------------------------
# decode workload
# ---------------------------------------------------------------------------

def decode_step_bytes(dec, pos):
    """Algorithmic HBM bytes of one decode step on this rank: every quantized
    weight once, the KV cache read (pos+1 positions) and the new K/V written."""
    cfg = dec.cfg
    kv_read = cfg.n_layers * dec.B * dec.hkv * (pos + 1) * cfg.head_dim * 2 * 2
    return dec.weight_bytes + kv_read


def bench_decode(args, torch, vm, dev, rank, world, grp=None):
    hbm, tf, tf_s, peak_src = peaks()
    cfg = vm.llama.LlamaConfig(n_layers=args.layers)
    B, ctx = args.batch, args.ctx
    pos = ctx  # the step appends token ctx+1 after `ctx` random cached tokens
    vm.lib().vmlx_set_launch_overlap(1)
    # TP: o_proj / down_proj run as fused GEMV + P2P all-reduce + residual kernels (group=grp)
    dec = vm.llama.LlamaDecoder(cfg, B, max_len=ctx + 8, dev=dev, seed=0, rank=rank, world=world,
                                group=grp, cache_fill=ctx)
    stream = torch.cuda.Stream(dev)
    x0 = torch.randn(B, cfg.hidden, device=dev, generator=torch.Generator(device=dev).manual_seed(3)).bfloat16()
    x = x0.clone()
    g = dec.capture(x, pos, stream)
    # the clock sampler runs from the warm-up through the GEMV-only timing below, so the line
    # carries its own samples even when the timed steps last less than one sampling period
    clk = ClockSampler(dev.index or 0).__enter__()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            g.replay()
        stream.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev[0].record(stream)
        for i in range(args.steps):
            g.replay()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    per_step = [ev[i].elapsed_time(ev[i + 1]) / 1e3 for i in range(args.steps)]
    t_mean = ev[0].elapsed_time(ev[-1]) / 1e3 / args.steps
    t_step = statistics.median(per_step)  # the reference's statistic (median of the steps)
    if world > 1:
        t = torch.tensor([t_step, t_mean], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_step, t_mean = t[0].item(), t[1].item()
    nbytes = decode_step_bytes(dec, pos)

    # dominant kernel: the quantized GEMV; time the step's GEMVs alone (same weights, same graph style)
    gemv_calls = []
    for L in dec.layers:
        gemv_calls += [lambda L=L: L.qkv(dec.h, out=dec.qkv_buf), lambda L=L: L.o(dec.attn.view(B, -1), out=dec.proj),
                       lambda L=L: L.gate_up(dec.h, out=dec.gu), lambda L=L: L.down(dec.act, out=dec.proj)]
    t_gemv = time_graph_calls(torch, gemv_calls, 5, 3, stream)
    gemv_bytes_avg = (dec.weight_bytes + len(gemv_calls) * B * 2 * (cfg.hidden + dec.ffn)) / len(gemv_calls)
    gemv_achieved = gemv_bytes_avg / t_gemv / 1e9

    # TP: the fused row-parallel kernels (GEMV + all-reduce + residual) alone, in lockstep on every rank
    tp_fused = None
    if grp is not None:
        racc = torch.zeros(B, cfg.hidden, dtype=torch.bfloat16, device=dev)
        tp_calls = []
        for L in dec.layers:
            tp_calls += [lambda L=L: grp.quantized_matmul_all_sum(dec.attn.view(B, -1), L.o, residual=racc, out=racc),
                         lambda L=L: grp.quantized_matmul_all_sum(dec.act, L.down, residual=racc, out=racc)]
        t_tp = time_graph_calls(torch, tp_calls, 5, 3, stream)
        # the same step through the plain GEMV + the unfused P2P all_sum + add, and with NCCL
        # all_reduce (the baseline the fused kernel replaces), graph-captured alike
        part = torch.empty(B, cfg.hidden, dtype=torch.bfloat16, device=dev)
        unf_calls, nccl_calls = [], []
        for L in dec.layers:
            for (xin, lin) in ((dec.attn.view(B, -1), L.o), (dec.act, L.down)):
                unf_calls += [lambda xin=xin, lin=lin: lin(xin, out=part),
                              lambda: grp.all_sum(part, out=part),
                              lambda: racc.add_(part)]
                nccl_calls += [lambda xin=xin, lin=lin: lin(xin, out=part),
                               lambda: torch.distributed.all_reduce(part),
                               lambda: racc.add_(part)]
        t_unf = time_graph_calls(torch, unf_calls, 5, 3, stream) * 3
        try:
            t_nccl = time_graph_calls(torch, nccl_calls, 5, 3, stream) * 3
        except Exception:  # NCCL graph capture unavailable: time it eagerly
            t_nccl = None
        t = torch.tensor([t_tp, t_unf, t_nccl or 0.0], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_tp, t_unf, t_nccl = t[0].item(), t[1].item(), (t[2].item() or None)
        w_tp = sum(L.o.nbytes + L.down.nbytes for L in dec.layers) / len(tp_calls)
        link = (world - 1) * B * cfg.hidden * 2  # bf16 partial rows sent to the other ranks per call
        t_target = max(w_tp / (hbm * 1e9), link / 770e9)
        tp_fused = {"kernel": "qgemv_kernel / qmv_kernel with the row-parallel all-reduce "
                              "(vmlx_tp_quantized_matmul_all_sum)",
                    "us_per_call": round(t_tp * 1e6, 2), "weight_bytes_per_call": int(w_tp),
                    "nvlink_bytes_out_per_call": link,
                    "unfused_us_per_call": round(t_unf * 1e6, 2),
                    "nccl_us_per_call": round(t_nccl * 1e6, 2) if t_nccl else None,
                    "nccl_baseline": "quantized GEMV + torch.distributed.all_reduce (NCCL) + residual add",
                    "roofline_us": round(t_target * 1e6, 2), "frac_of_combined_roofline": round(t_target / t_tp, 4),
                    "roofline_basis": "max(weight bytes / measured HBM, NVLink bytes / 770 GB/s measured peer copy)"}

    clk.__exit__(None, None, None)
    # end to end through the public API: host token state in, host state out, every step
    xh = x0.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    n_e2e = max(8, args.steps // 2)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(n_e2e):
            dec.decode(xh, out=yh)
        e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3 / n_e2e
    res = {
        "metric": "decode tokens/s (Llama-3-8B-shaped decoder, 4-bit g64, TP=N)",
        "value": round(B / t_step, 2), "unit": "tokens/s", "higher_is_better": True,
        "ms_per_step": t_step * 1e3, "ms_per_step_mean": round(t_mean * 1e3, 4), "step_statistic": "median",
        "dtype": "bf16",
        "config": {"workload": f"BASELINE config 3: {cfg.n_layers} Llama-3-8B-shaped blocks (hidden 4096, "
                               f"32 Q / 8 KV heads, hd 128, FFN 14336, 4-bit g64), batch {B}, bf16 KV cache of "
                               f"{ctx} random tokens, TP={world}",
                   "batch": B, "context": ctx, "layers": cfg.n_layers, "parallelism": f"tp{world}",
                   "l2": f"inputs larger than L2: {nbytes / 1e9:.2f} GB of weights + KV per step per rank",
                   "graph": "whole decode step captured in one CUDA graph", "launch_overlap": "on"},
        "step_hbm": {"bytes_per_rank": nbytes, "GBps_per_rank": round(nbytes / t_step / 1e9, 1),
                     "frac_of_measured": round(nbytes / t_step / 1e9 / hbm, 4)},
        "roofline": {"bound": "hbm", "kernel": "decode GEMVs (qgemv_kernel up to 8K x 8K, qmv_kernel above)", "achieved": round(gemv_achieved, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(gemv_achieved / hbm, 4), "peak_source": peak_src,
                     "frac_of_8TBps": round(gemv_achieved / 8000, 4),
                     "traffic": load_traffic(f"decode_gemvs_B{B}_tp{world}"),
                     "algorithmic_bytes_per_launch": int(gemv_bytes_avg), "us_per_launch": round(t_gemv * 1e6, 2)},
        "e2e": {"value": round(B / t_e2e, 2), "unit": "tokens/s", "ms_per_step": round(t_e2e * 1e3, 3),
                "h2d_bytes_per_step": B * cfg.hidden * 2, "d2h_bytes_per_step": B * cfg.hidden * 2},
        "gpu_launches": args.steps * dec.launches_per_step,
        **({"tp_fused": tp_fused} if tp_fused else {}),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        res["cpu_baseline"] = cpu_baseline_decode(B, ctx, cfg, seconds=args.cpu_seconds)
    if args.profile:  # one eager decode step inside an NVTX range (ncu --nvtx-include vmlx_profile/)
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("vmlx_profile")
            dec.step(x, pos)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    return res


def bench_qwen3(args, torch, vm, dev):
    """Qwen3-32B-shaped greedy generation (64 layers, 4-bit g64, vocab 151936).
    The prompt (args.ctx token ids, uniform over the vocabulary) is prefilled untimed; a step is
    one generated token per sequence: embedding, 64 blocks, lm_head, argmax, all in one CUDA graph
    that reads and advances the position on the device."""
    hbm, tf, tf_s, peak_src = peaks()
    cfg = vm.qwen3.Qwen3Config(n_layers=args.layers if args.layers != 32 else 64)
    B, T = args.batch, args.ctx if args.ctx != 4096 else 2048
    vm.lib().vmlx_set_launch_overlap(1)
    n_e2e = max(8, args.steps // 2)
    max_len = T + max(3, args.warmup) + args.steps + n_e2e + 16  # every replayed step appends one position
    dec = vm.qwen3.Qwen3Decoder(cfg, B, max_len=max_len, dev=dev, seed=0)
    prompt = torch.randint(0, cfg.vocab, (B, T), device=dev, generator=torch.Generator(device=dev).manual_seed(1))
    t0 = time.perf_counter()
    dec.prefill(prompt)
    torch.cuda.synchronize()
    t_prefill = time.perf_counter() - t0
    stream = torch.cuda.Stream(dev)
    g = dec.capture(stream)
    clk = ClockSampler(dev.index or 0).__enter__()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            g.replay()
        stream.synchronize()
        ev[0].record(stream)
        for i in range(args.steps):
            g.replay()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    per_step = [ev[i].elapsed_time(ev[i + 1]) / 1e3 for i in range(args.steps)]
    t_step = statistics.median(per_step)
    ctx_mid = T + max(3, args.warmup) + args.steps // 2
    kv_bytes = cfg.n_layers * B * cfg.n_kv_heads * ctx_mid * cfg.head_dim * 2 * 2
    nbytes = dec.weight_bytes + kv_bytes
    # dominant kernels: the step's quantized GEMVs (4 per block + lm_head), timed alone in a graph
    x = torch.randn(B, cfg.hidden, device=dev).bfloat16()
    calls = []
    for L in dec.layers:
        calls += [lambda L=L: L.qkv(x, out=dec.qkv_buf), lambda L=L: L.o(dec.attn.view(B, -1), out=dec.proj),
                  lambda L=L: L.gate_up(x, out=dec.gu), lambda L=L: L.down(dec.act, out=dec.proj)]
    calls.append(lambda: dec.lm_head(x, out=dec.logits))
    t_gemv = time_graph_calls(torch, calls, 3, 2, stream)
    gemv_bytes = sum(l.nbytes for l in dec.layers) + dec.lm_head.nbytes
    gemv_bytes_avg = gemv_bytes / len(calls)
    clk.__exit__(None, None, None)
    # end to end: the sampled ids to the host and the next step's ids from the host, every step
    ids_h = torch.empty(B, dtype=torch.int32).pin_memory()
    ids_h.copy_(dec.ids.cpu())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(n_e2e):
            dec.ids.copy_(ids_h, non_blocking=True)
            g.replay()
            ids_h.copy_(dec.ids, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1) / 1e3 / n_e2e
    if args.profile:  # one eager decode step inside an NVTX range (ncu --nvtx-include vmlx_profile/)
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("vmlx_profile")
            dec.step()
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    return {
        "metric": "decode tokens/s (Qwen3-32B-shaped greedy generation, 4-bit g64)",
        "value": round(B / t_step, 2), "unit": "tokens/s", "higher_is_better": True,
        "ms_per_step": t_step * 1e3, "step_statistic": "median", "dtype": "bf16",
        "config": {"workload": f"BASELINE config 5: {cfg.n_layers} Qwen3-32B-shaped blocks (hidden 5120, 64 Q / 8 "
                               f"KV heads, hd 128, FFN 25600, vocab 151936, 4-bit g64), batch {B}, prompt {T} "
                               f"uniform ids prefilled untimed, greedy decode steps, TP=1",
                   "batch": B, "prompt": T, "layers": cfg.n_layers, "parallelism": "tp1",
                   "prefill_s": round(t_prefill, 2),
                   "l2": f"inputs larger than L2: {nbytes / 1e9:.2f} GB of weights + KV per step",
                   "graph": "one CUDA graph per token (device-side position), replayed", "launch_overlap": "on"},
        "step_hbm": {"bytes": nbytes, "GBps": round(nbytes / t_step / 1e9, 1),
                     "frac_of_measured": round(nbytes / t_step / 1e9 / hbm, 4)},
        "roofline": {"bound": "hbm", "kernel": "decode GEMVs (qgemv_kernel / qmv_kernel) incl. lm_head",
                     "achieved": round(gemv_bytes_avg / t_gemv / 1e9, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gemv_bytes_avg / t_gemv / 1e9 / hbm, 4), "peak_source": peak_src,
                     "traffic": load_traffic(f"qwen3_gemvs_B{B}_{cfg.n_layers}layers"),
                     "algorithmic_bytes_per_launch": int(gemv_bytes_avg),
                     "us_per_launch": round(t_gemv * 1e6, 2)},
        "e2e": {"value": round(B / t_e2e, 2), "unit": "tokens/s", "ms_per_step": round(t_e2e * 1e3, 3),
                "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * 4},
        "gpu_launches": args.steps * dec.launches_per_step,
        "status": int(dec.status.item()),
        "clocks": clk.summary(),
    }


def cpu_baseline_decode(B, ctx, cfg, seconds=10.0):
    """CPU restatement of one decode step (oracle GEMVs of one layer + numpy
    attention over the cache), timed over whole layers and scaled to the stack."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    rng = np.random.default_rng(0)
    H, D, Hq, Hkv, F = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn

    def qw(n, k):
        return oracle.quantize(oracle.f32_to_bf16(rng.normal(0, 0.02, (n, k)).astype(np.float32)), 64, 4)
    mats = [((Hq + 2 * Hkv) * D, H), (H, Hq * D), (2 * F, H), (H, F)]
    ws = [qw(n, k) for n, k in mats]
    kc = rng.normal(size=(B, Hkv, ctx + 1, D)).astype(np.float32)
    vc = rng.normal(size=(B, Hkv, ctx + 1, D)).astype(np.float32)
    xs = [oracle.f32_to_bf16(rng.normal(size=(B, k)).astype(np.float32)) for _, k in mats]
    q = rng.normal(size=(B, Hq, D)).astype(np.float32)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds or n == 0:
        for (wq, s, b), x in zip(ws, xs):
            oracle.qmm_fp32_bf16(x, wq, s, b, 64, 4)
        G = Hq // Hkv
        sc = np.einsum("bhgd,bhtd->bhgt", q.reshape(B, Hkv, G, D), kc) * D ** -0.5
        p = np.exp(sc - sc.max(-1, keepdims=True))
        np.einsum("bhgt,bhtd->bhgd", p / p.sum(-1, keepdims=True), vc)
        n += 1
    dt_layer = (time.perf_counter() - t0) / n
    t_tok = dt_layer * cfg.n_layers
    return {"value": round(B / t_tok, 4), "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n} layer steps (4 quantized GEMVs via the OpenMP C restatement + numpy attention over "
                      f"{ctx + 1} cached tokens) in {seconds:.0f} s, scaled to {cfg.n_layers} layers",
            "ms_per_token": round(t_tok * 1e3, 2)}


# ---------------------------------------------------------------------------
# driver
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=os.environ.get("VMLX_BENCH_WORKLOAD", "decode"),
                    choices=["gemv", "decode", "moe", "qwen3"])
    ap.add_argument("--quick", action="store_true", help="skip the config-2 sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=1, help="decode batch (config 3: 1, 16, 64)")
    ap.add_argument("--ctx", type=int, default=4096, help="cached tokens before the step")
    ap.add_argument("--layers", type=int, default=32, help="decoder blocks (Llama-3-8B has 32)")
    ap.add_argument("--tokens", type=int, default=32, help="MoE workload: tokens per layer (config 4: 1, 32, 256)")
    ap.add_argument("--profile", action="store_true",
                    help="after timing, run one eager instance of the profiled kernels in NVTX range vmlx_profile")
    args = ap.parse_args()
    rank, world, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        line = reference_arm(args, world)
        print(json.dumps(line), flush=True)
        return

    import torch
    from vmlx_b200_loader import load_package
    vm = load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.workload == "moe":
        grp = vm.distributed.Group(strict=True) if world > 1 else None
        res = bench_moe(args, torch, vm, dev, grp)
        if grp is not None:
            res["tp_status"] = grp.status()
        res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "scaling": "strong",
                    "vs_baseline": None, "data": "synthetic (seeded random experts, router logits and tokens)"})
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    if args.workload == "qwen3":
        if world > 1:
            raise SystemExit("the qwen3 workload runs at TP=1 (the tensor-parallel path is the decode workload)")
        res = bench_qwen3(args, torch, vm, dev)
        res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "scaling": "strong",
                    "vs_baseline": None, "data": "synthetic (seeded random-init quantized weights and prompt ids)"})
        print(json.dumps(res), flush=True)
        return
    if args.workload == "gemv":
        if world > 1:
            # the single-matrix GEMV does not shard: N independent replicas
            import torch.distributed as dist
            dist.init_process_group("nccl", device_id=dev)
        res = bench_gemv(args, torch, vm, dev)
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([res["ms_per_step"]], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res["ms_per_step"] = t.item()
            res["value"] = round(res["value"] * world, 1)  # replicas: whole-job bytes/s
            dist.destroy_process_group()
        res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "scaling": "weak", "vs_baseline": None, "data": "synthetic (seeded torch RNG)"})
        res["config"]["parallelism"] = f"replicas{world}" if world > 1 else "single"
        if rank == 0:
            print(json.dumps(res), flush=True)
    else:
        grp = None
        if world > 1:
            # one rank per GPU: P2P all-reduce group bootstrapped over torch.distributed (NCCL only for the bootstrap)
            grp = vm.distributed.Group(strict=True)
        res = bench_decode(args, torch, vm, dev, rank, world, grp)
        if grp is not None:
            res["tp_status"] = grp.status()
        res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "scaling": "strong",
                    "vs_baseline": None, "data": "synthetic (seeded random weights, tokens and KV cache)"})
        if rank == 0:
            print(json.dumps(res), flush=True)


def reference_arm(args, world):
    """The reference's own CPU path for this workload (MLX's CPU code is absent
    from the reference checkout, so: the C restatement of its arithmetic)."""
    note = ("reference CPU path = C restatement of MLX's affine qmv (MLX's own CPU code is absent from the "
            "reference checkout)")
    if args.workload == "decode":
        sys.path.insert(0, ROOT)
        from vmlx_b200_loader import load_package
        vm = load_package()
        cfg = vm.llama.LlamaConfig(n_layers=args.layers)
        cpu = cpu_baseline_decode(args.batch, args.ctx, cfg, seconds=args.cpu_seconds)
        return {"impl": "reference", "metric": "decode tokens/s (Llama-3-8B-shaped decoder, 4-bit g64, TP=N)",
                "value": cpu["value"], "unit": "tokens/s", "higher_is_better": True, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": cpu["ms_per_token"], "dtype": "bf16",
                "data": "synthetic (seeded numpy PCG64)", "scaling": "strong", "vs_baseline": None,
                "config": {"workload": f"BASELINE config 3: {cfg.n_layers} Llama-3-8B-shaped blocks, batch "
                                       f"{args.batch}, {args.ctx} cached tokens", "batch": args.batch,
                           "context": args.ctx, "layers": cfg.n_layers, "note": note},
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    M, N, K, bits, gs = 1, 4096, 4096, 4, 64
    cpu = cpu_baseline_gemv(M, N, K, bits, gs, seconds=args.cpu_seconds)
    return {"impl": "reference", "metric": "quantized GEMV HBM GB/s (4096x4096, 4-bit g64, M=1)",
            "value": cpu["value"], "unit": "GB/s", "higher_is_better": True, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cpu["us_per_call"] / 1e3,
            "dtype": "bf16", "data": "synthetic (seeded numpy PCG64)", "scaling": "weak", "vs_baseline": None,
            "config": {"workload": "BASELINE config 1: MLX affine quantized_matmul GEMV", "M": M, "N": N, "K": K,
                       "bits": bits, "group_size": gs, "note": note},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


if __name__ == "__main__":
    main()
