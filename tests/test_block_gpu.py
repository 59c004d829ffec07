"""GPU parity of the decoder-block support kernels and of a whole decode step
against numpy references (fp64 math, the reference's bf16 rounding points).
Tolerance as for the matmuls: max |err| / max |ref| <= 1e-2 and mean
|err - bf16 rounding| / mean |ref| <= 1e-3 (looser 3e-3 where several bf16
roundings compound across a whole layer)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def f(t):
    return t.float().cpu().numpy().astype(np.float64)


def check(got, ref, max_rel=1e-2, mean_rel=1e-3):
    import oracle
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    ref16 = oracle.round_bf16(ref.astype(np.float32)).astype(np.float64)
    assert np.abs(got - ref).max() / (np.abs(ref).max() + 1e-30) <= max_rel
    assert np.abs(got - ref16).mean() / (np.abs(ref).mean() + 1e-30) <= mean_rel


def bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


bits_of16 = bits


@pytest.mark.parametrize("dims", [512, 4096, 5120])
def test_rms_norm(vm, orc, cuda, dims):
    g = torch.Generator(cuda).manual_seed(dims)
    x = (torch.randn(7, dims, device=cuda, generator=g) * 3).bfloat16()
    w = (1 + 0.1 * torch.randn(dims, device=cuda, generator=g)).bfloat16()
    y = vm.fast.rms_norm(x, w, 1e-5)
    ref = orc.rms_norm_ref(bits(x), bits(w), 1e-5)
    check(f(y), ref)
    # at most one bf16 ulp away from the reference's rounding order
    assert np.abs(f(y) - ref).max() <= np.abs(ref).max() * 2 ** -7


def test_rope_qkv_and_cache_append(vm, orc, cuda):
    B, Hq, Hkv, D, L, pos = 3, 8, 2, 128, 40, 29
    g = torch.Generator(cuda).manual_seed(1)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    kc = torch.zeros(B, Hkv, L, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = vm.fast.rope_qkv(qkv, kc, vc, Hq, Hkv, pos, base=500000.0)
    x = f(qkv).reshape(B, Hq + 2 * Hkv, D)
    check(f(q), orc.rope_ref(x[:, :Hq], pos, 500000.0))
    check(f(kc[:, :, pos]), orc.rope_ref(x[:, Hq:Hq + Hkv], pos, 500000.0))
    assert torch.equal(vc[:, :, pos], qkv.view(B, Hq + 2 * Hkv, D)[:, Hq + Hkv:])
    assert torch.count_nonzero(kc[:, :, :pos]) == 0  # nothing else written


@pytest.mark.parametrize("kv_len,G", [(1, 4), (37, 1), (300, 4), (4097, 4), (700, 8)])
def test_sdpa_decode(vm, orc, cuda, kv_len, G):
    B, Hkv, D = 2, 2, 128
    Hq = Hkv * G
    L = kv_len + 5
    g = torch.Generator(cuda).manual_seed(kv_len)
    q = torch.randn(B, Hq, D, device=cuda, generator=g).bfloat16()
    kc = torch.randn(B, Hkv, L, D, device=cuda, generator=g).bfloat16()
    vc = torch.randn(B, Hkv, L, D, device=cuda, generator=g).bfloat16()
    o = vm.fast.sdpa_decode(q, kc, vc, kv_len)
    ref = orc.sdpa_ref(f(q), f(kc)[:, :, :kv_len], f(vc)[:, :, :kv_len], D ** -0.5)
    check(f(o), ref)


def test_silu_mul_and_add(vm, orc, cuda):
    g = torch.Generator(cuda).manual_seed(3)
    gu = (torch.randn(5, 2 * 768, device=cuda, generator=g) * 2).bfloat16()
    a = vm.fast.silu_mul(gu)
    gg, uu = f(gu)[:, :768], f(gu)[:, 768:]
    s = orc.round_bf16((gg / (1 + np.exp(-gg))).astype(np.float32)).astype(np.float64)
    check(f(a), s * uu)
    x, y = gu[:, :768].contiguous(), gu[:, 768:].contiguous()
    assert torch.equal(vm.fast.add(x, y), (x.float() + y.float()).bfloat16())


def _layer_ref(orc, dec, x, pos):
    """numpy restatement of LlamaDecoder.step (TP=1) with its bf16 rounding points."""
    cfg = dec.cfg
    B = x.shape[0]
    r16 = lambda a: orc.round_bf16(np.asarray(a, np.float32)).astype(np.float64)  # noqa: E731
    b16 = lambda a: orc.f32_to_bf16(np.asarray(a, np.float32))  # noqa: E731

    def qmm(a, ql):
        wq = ql.wq.cpu().numpy().view(np.uint32)
        return r16(orc.qmm_f64(b16(a), wq, bits(ql.scales), bits(ql.biases), cfg.group_size, cfg.bits))

    x = x.astype(np.float64)
    D, Hq, Hkv = cfg.head_dim, dec.hq, dec.hkv
    for i, Lw in enumerate(dec.layers):
        h = orc.rms_norm_ref(b16(x), bits(Lw.norm1), cfg.eps)
        qkv = qmm(h, Lw.qkv).reshape(B, Hq + 2 * Hkv, D)
        q = r16(orc.rope_ref(qkv[:, :Hq], pos, cfg.rope_theta))
        k_new = r16(orc.rope_ref(qkv[:, Hq:Hq + Hkv], pos, cfg.rope_theta))
        kc = f(dec.k_cache[i]).copy()
        vc = f(dec.v_cache[i]).copy()
        kc[:, :, pos] = k_new
        vc[:, :, pos] = qkv[:, Hq + Hkv:]
        a = r16(orc.sdpa_ref(q, kc[:, :, :pos + 1], vc[:, :, :pos + 1], D ** -0.5))
        o = qmm(a.reshape(B, -1), Lw.o)
        x = r16(x + o)
        h2 = orc.rms_norm_ref(b16(x), bits(Lw.norm2), cfg.eps)
        gu = qmm(h2, Lw.gate_up)
        F = gu.shape[1] // 2
        act = r16(r16(gu[:, :F] / (1 + np.exp(-gu[:, :F]))) * gu[:, F:])
        x = r16(x + qmm(act, Lw.down))
    return x


@pytest.mark.parametrize("fused,B", [(False, 3), (True, 3), (False, 16), (True, 16), (True, 64)])
def test_decoder_step_matches_reference(vm, orc, cuda, fused, B):
    """BASELINE config 3 batches (1/16/64; B=64 runs the tensor-core GEMM for every linear)."""
    cfg = vm.llama.LlamaConfig(hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, n_layers=2)
    pos = 64
    dec = vm.llama.LlamaDecoder(cfg, B, max_len=96, dev=cuda, seed=5, cache_fill=pos, fused=fused)
    g = torch.Generator(cuda).manual_seed(9)
    x = torch.randn(B, cfg.hidden, device=cuda, generator=g).bfloat16()
    x0 = f(x)
    ref = _layer_ref(orc, dec, x0, pos)  # reads the caches before the step mutates them
    y = dec.step(x, pos)
    check(f(y), ref, max_rel=2e-2, mean_rel=3e-3)


def test_decoder_step_cuda_graph_replay(vm, orc, cuda):
    """The decode step is capture-safe: a replayed graph equals an eager step."""
    cfg = vm.llama.LlamaConfig(hidden=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, n_layers=2)
    dec = vm.llama.LlamaDecoder(cfg, 2, max_len=64, dev=cuda, seed=2, cache_fill=32)
    x0 = torch.randn(2, cfg.hidden, device=cuda).bfloat16()
    x = x0.clone()
    eager = dec.step(x, 32).clone()
    st = torch.cuda.Stream()
    xg = x0.clone()
    with torch.cuda.stream(st):
        dec.step(xg.copy_(x0), 32)
        st.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=st):
            dec.step(xg, 32)
        xg.copy_(x0)
        gph.replay()
    torch.cuda.synchronize()
    assert torch.equal(xg, eager)


@pytest.mark.parametrize("M", [1, 4, 9])
def test_fused_gemv_matches_separate_kernels(vm, orc, cuda, M):
    """RMSNorm-on-load and residual-on-store fusions equal the separate kernels
    up to the last bit of 1/rms (tolerance) for 4-bit (CUDA-core and MMA paths) and 8-bit."""
    K, N = 2048, 512
    g = torch.Generator(cuda).manual_seed(M)
    for bits in (4, 8):
        w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
        wq, s, b = vm.quantized(w, bits=bits)
        x = (torch.randn(M, K, device=cuda, generator=g) * 2).bfloat16()
        nw = (1 + 0.1 * torch.randn(K, device=cuda, generator=g)).bfloat16()
        res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
        xn = vm.fast.rms_norm(x, nw, 1e-5)
        got = vm.ops.quantized_mm_fused(x, wq, s, b, bits=bits, norm_weight=nw, eps=1e-5, residual=res)
        if M <= 4:  # the separate quantized_mm runs the same GEMV kernels
            ref = vm.fast.add(res, vm.quantized_mm(xn, wq, s, b, bits=bits))
            check(f(got), f(ref))
        else:  # quantized_mm runs the tcgen05 GEMM from 5 rows: hold the fused GEMV to the fp64 oracle
            xb = xn.cpu().view(torch.int16).numpy().view(np.uint16)
            exact = orc.qmm_f64(xb, wq.cpu().numpy().view(np.uint32), bits_of16(s), bits_of16(b), 64, bits)
            check(f(got), f(res) + orc.round_bf16(exact.astype(np.float32)).astype(np.float64), mean_rel=2e-3)
        y = res.clone()
        vm.ops.quantized_mm_fused(x, wq, s, b, bits=bits, norm_weight=nw, residual=y, out=y)  # in place
        assert torch.equal(y, got)


@pytest.mark.parametrize("M", [1, 4, 9])
def test_swiglu_fused_down_gemv_matches_separate_kernels(vm, orc, cuda, M):
    """The SwiGLU computed while the down GEMV stages x rounds exactly as silu_mul: the fused
    call equals silu_mul -> quantized_mm (-> add) bit for bit (4-bit CUDA-core and MMA paths, 8-bit)."""
    K, N = 1536, 512
    g = torch.Generator(cuda).manual_seed(10 + M)
    for bits in (4, 8):
        w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
        wq, s, b = vm.quantized(w, bits=bits)
        gu = (torch.randn(M, 2 * K, device=cuda, generator=g) * 2).bfloat16()
        res = torch.randn(M, N, device=cuda, generator=g).bfloat16()
        act = vm.fast.silu_mul(gu)
        sep = vm.quantized_mm(act, wq, s, b, bits=bits) if M <= 4 else vm.ops.quantized_mm_fused(act, wq, s, b, bits=bits)
        assert torch.equal(vm.ops.quantized_mm_swiglu(gu, wq, s, b, bits=bits), sep)
        ref = vm.ops.quantized_mm_fused(act, wq, s, b, bits=bits, residual=res)
        y = res.clone()
        vm.ops.quantized_mm_swiglu(gu, wq, s, b, bits=bits, residual=y, out=y)
        assert torch.equal(y, ref)
