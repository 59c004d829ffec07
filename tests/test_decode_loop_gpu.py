"""GPU tests of the decode-loop pieces around the linears (csrc/decode.cu, the device-position
attention entry point) and of the Qwen3 greedy token loop built from them, through the C ABI.

Bars: the quantized embedding is bit-exact against dequantize of the gathered rows (the same
bf16 arithmetic); RoPE with the per-head q/k RMSNorm matches a float64 restatement within bf16
rounding, and gives the same bits whether the position comes from device memory or an int and
whether rows are decoded one position at a time or prefilled together; attention with the cache
length read on the device equals attention given the length; greedy sampling equals numpy's
argmax (first index of the maximum); a replayed token-loop graph produces the same tokens as
eager steps; the decode step's logits match a float32 recompute of the whole sequence with the
dequantized weights."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_quantized_embedding_bit_exact(vm, cuda):
    g = torch.Generator(cuda).manual_seed(0)
    V, H = 1000, 512
    w = (torch.randn(V, H, device=cuda, generator=g) * 0.02).bfloat16()
    for bits in (4, 8):
        wq, s, b = vm.quantized(w, group_size=64, bits=bits)
        ids = torch.tensor([0, 7, 999, 7, 512], dtype=torch.int32, device=cuda)
        out = vm.fast.quantized_embedding(ids, wq, s, b, 64, bits)
        ref = vm.dequantized(wq[ids.long()], s[ids.long()], b[ids.long()], group_size=64, bits=bits)
        assert torch.equal(out, ref)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    bad = vm.fast.quantized_embedding(torch.tensor([3, V], dtype=torch.int32, device=cuda), wq, s, b, 64, 8,
                                      status=st)
    torch.cuda.synchronize()
    assert st.item() == vm._lib.VMLX_E_INVALID and torch.count_nonzero(bad[1]) == 0


def _rope_ref(qkv, Hq, Hkv, D, pos, qn, kn, eps, base):
    """float64 restatement with the kernel's bf16 roundings: RMSNorm per head, then RoPE."""
    x = qkv.double().view(qkv.shape[0], Hq + 2 * Hkv, D)
    heads = x[:, :Hq + Hkv].clone()
    w = torch.cat([qn.double().expand(Hq, D), kn.double().expand(Hkv, D)], 0)
    inv = torch.rsqrt((heads * heads).mean(-1, keepdim=True) + eps)
    n = (heads * inv).float().bfloat16().double()
    heads = (w * n).float().bfloat16().double()
    half = D // 2
    d = torch.arange(half, dtype=torch.float64, device=qkv.device)
    inv_freq = base ** (-d / half)
    th = pos.double().view(-1, 1, 1) * inv_freq
    x1, x2 = heads[..., :half], heads[..., half:]
    rot = torch.cat([x1 * th.cos() - x2 * th.sin(), x1 * th.sin() + x2 * th.cos()], -1)
    return rot[:, :Hq], rot[:, Hq:], x[:, Hq + Hkv:]


def test_rope_qk_norm_decode_and_prefill(vm, cuda):
    g = torch.Generator(cuda).manual_seed(1)
    Hq, Hkv, D, T, L = 8, 2, 128, 5, 16
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda, generator=g).bfloat16() * 2
    qn = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).bfloat16()
    kn = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).bfloat16()
    kc = torch.zeros(1, Hkv, L, D, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    # prefill: rows 0..T-1 are positions 3..3+T-1 of sequence 0
    q = vm.fast.rope_qk_norm(qkv, kc, vc, Hq, Hkv, 3, qn, kn, 1e-6, 1e6, tokens_per_seq=T)
    qr, kr, vr = _rope_ref(qkv, Hq, Hkv, D, torch.arange(3, 3 + T, device=cuda), qn, kn, 1e-6, 1e6)
    assert (q.double() - qr).abs().max().item() <= 2e-2 * qr.abs().max().item()
    assert (kc[0, :, 3:3 + T].transpose(0, 1).double() - kr).abs().max().item() <= 2e-2 * kr.abs().max().item()
    assert torch.equal(vc[0, :, 3:3 + T].transpose(0, 1), vr.bfloat16())
    # decode, one row at a time with the position on the device: the same bits
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    for t in range(T):
        pos.fill_(3 + t)
        qt = vm.fast.rope_qk_norm(qkv[t:t + 1], kc2, vc2, Hq, Hkv, pos, qn, kn, 1e-6, 1e6)
        assert torch.equal(qt[0], q[t])
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)
    # without the norms this is the Llama RoPE of rope_qkv
    kc3, vc3, kc4, vc4 = (torch.zeros_like(kc) for _ in range(4))
    a = vm.fast.rope_qk_norm(qkv[:1], kc3, vc3, Hq, Hkv, 7, base=5e5)
    b = vm.fast.rope_qkv(qkv[:1], kc4, vc4, Hq, Hkv, 7, base=5e5)
    assert (a.float() - b.float()).abs().max().item() <= 1e-2 * b.float().abs().max().item()
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    pos.fill_(L)  # past the cache: skipped, status set
    vm.fast.rope_qk_norm(qkv[:1], kc3, vc3, Hq, Hkv, pos, status=st)
    torch.cuda.synchronize()
    assert st.item() == vm._lib.VMLX_E_INVALID


def test_sdpa_decode_at_matches_host_length(vm, cuda):
    g = torch.Generator(cuda).manual_seed(2)
    B, Hq, Hkv, D, L = 2, 16, 4, 128, 1100
    q = torch.randn(B, Hq, D, device=cuda, generator=g).bfloat16()
    kc = torch.randn(B, Hkv, L, D, device=cuda, generator=g).bfloat16()
    vc = torch.randn(B, Hkv, L, D, device=cuda, generator=g).bfloat16()
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws = torch.zeros(vm.fast.sdpa_workspace_bytes(B, Hq, L, D), dtype=torch.uint8, device=cuda)
    for kv_len in (1, 255, 256, 257, 700, L):
        pos.fill_(kv_len - 1)
        a = vm.fast.sdpa_decode_at(q, kc, vc, pos, workspace=ws)
        b = vm.fast.sdpa_decode(q, kc, vc, kv_len)
        assert torch.equal(a, b), kv_len


def test_argmax_first_index(vm, cuda):
    g = torch.Generator(cuda).manual_seed(3)
    V = 151936
    x = torch.randn(5, V, device=cuda, generator=g).bfloat16()
    x[1, 100] = x[1, 90000] = 50.0  # a tie: the first index wins
    x[2] = -float("inf")
    x[2, V - 1] = 0.0
    x[3, 17] = float("nan")
    out = vm.fast.argmax(x).cpu().numpy()
    xs = x.float().cpu().numpy()
    xs = np.where(np.isnan(xs), -np.inf, xs)
    assert out.tolist() == np.argmax(xs, axis=1).tolist()


def _small_cfg(vm, layers=2):
    return vm.qwen3.Qwen3Config(hidden=512, n_heads=8, n_kv_heads=2, head_dim=128, ffn=1024, n_layers=layers,
                                vocab=1024)


def test_token_loop_graph_matches_eager_steps(vm, cuda):
    cfg = _small_cfg(vm)
    prompt = torch.randint(0, cfg.vocab, (2, 9), generator=torch.Generator().manual_seed(4)).to(cuda)
    runs = []
    for mode in ("eager", "graph"):
        dec = vm.qwen3.Qwen3Decoder(cfg, 2, max_len=64, dev=cuda, seed=5)
        first = dec.prefill(prompt).clone()
        if mode == "eager":
            toks = [dec.step().clone() for _ in range(12)]
            toks = torch.stack(toks).cpu()
        else:
            dec.capture()
            toks = dec.generate(12)
            torch.cuda.synchronize()  # generate() copies the ids to the host asynchronously
            toks = toks.clone()
        assert dec.pos.item() == 9 + 12 and dec.status.item() == 0
        runs.append((first.cpu(), toks))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])


def _fp32_forward(vm, dec, seq):
    """float32 recompute of the last position's logits for the token sequences seq [B, T] with
    the dequantized weights (no cache)."""
    cfg = dec.cfg
    Hq, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

    def deq(ql):
        return vm.dequantized(ql.wq, ql.scales, ql.biases, group_size=cfg.group_size, bits=cfg.bits).float()

    def rms(x, w):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.eps) * w.float()

    B, T = seq.shape
    emb = vm.dequantized(*dec.embed, group_size=cfg.group_size, bits=cfg.bits).float()
    x = emb[seq.long()]
    half = D // 2
    inv_freq = cfg.rope_theta ** (-torch.arange(half, device=seq.device, dtype=torch.float32) / half)
    th = (torch.arange(T, device=seq.device, dtype=torch.float32)[:, None] * inv_freq)[:, None, :]  # [T, 1, D/2]

    def rope(t):
        a, b = t[..., :half], t[..., half:]
        return torch.cat([a * th.cos() - b * th.sin(), a * th.sin() + b * th.cos()], -1)

    for L in dec.layers:
        qkv = rms(x, L.norm1) @ deq(L.qkv).T
        q = qkv[..., :Hq * D].view(B, T, Hq, D)
        k = qkv[..., Hq * D:(Hq + Hkv) * D].view(B, T, Hkv, D)
        v = qkv[..., (Hq + Hkv) * D:].view(B, T, Hkv, D)
        q, k = rope(rms(q, L.q_norm)).transpose(1, 2), rope(rms(k, L.k_norm)).transpose(1, 2)
        a = torch.nn.functional.scaled_dot_product_attention(q, k, v.transpose(1, 2), is_causal=True,
                                                             enable_gqa=True)
        x = x + a.transpose(1, 2).reshape(B, T, -1) @ deq(L.o).T
        gu = rms(x, L.norm2) @ deq(L.gate_up).T
        gt, up = gu[..., :cfg.ffn], gu[..., cfg.ffn:]
        x = x + (torch.nn.functional.silu(gt) * up) @ deq(L.down).T
    return rms(x[:, -1], dec.final_norm) @ deq(dec.lm_head).T


@pytest.mark.parametrize("B", [1, 8])
def test_decode_logits_match_fp32_recompute(vm, cuda, B):
    cfg = _small_cfg(vm)
    dec = vm.qwen3.Qwen3Decoder(cfg, B, max_len=48, dev=cuda, seed=6)
    prompt = torch.randint(0, cfg.vocab, (B, 7), generator=torch.Generator().manual_seed(7)).to(cuda)
    ids = dec.prefill(prompt).clone()
    seq = torch.cat([prompt.to(torch.int32), ids[:, None]], 1)
    ref = _fp32_forward(vm, dec, seq)
    dec.step()
    got = dec.logits.float()
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    assert err <= 5e-2, err
