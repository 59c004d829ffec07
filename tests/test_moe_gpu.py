"""MoE routing on the device: routing (Qwen3MoE.swift:137-148), gatherSort /
scatterUnsort (SwitchLayers.swift:64-83), the score-weighted combine
(Qwen3MoE.swift:150-151), and SwitchGLU / the whole block at BASELINE config 4
(hidden 2048, 128 experts, FFN 768, top-8) against the oracle."""
import numpy as np
import pytest
import torch

from test_quant_gpu import bits_of, check_close, make_weights, to_dev_bf16, u32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (32, 128, 8), (256, 128, 8), (7, 60, 4), (3, 1000, 32)])
@pytest.mark.parametrize("norm", [False, True])
def test_moe_route_matches_oracle(vm, orc, cuda, T, E, k, norm):
    rng = np.random.default_rng(T * 1000 + E + k)
    logits = rng.normal(0, 1, (T, E)).astype(np.float32)
    inds, scores = vm.ops.moe_route(torch.from_numpy(logits).to(cuda), k, norm)
    inds = inds.cpu().numpy().astype(np.int64)
    scores = scores.cpu().numpy()
    ref_inds, ref_scores = orc.moe_route(logits, k, norm)
    # the same expert sets; ours in descending logit order
    assert np.array_equal(np.sort(inds, -1), ref_inds)
    assert np.all(np.diff(np.take_along_axis(logits, inds, -1), axis=-1) <= 0)
    got = np.take_along_axis(scores, np.argsort(inds, -1), -1)
    np.testing.assert_allclose(got, ref_scores, rtol=2e-6, atol=1e-9)


def test_moe_route_bf16_and_ties(vm, orc, cuda):
    """bf16 logits (ties are common): scores in bf16, ids by descending logit then id."""
    logits = torch.zeros(4, 128, device=cuda, dtype=torch.bfloat16)
    logits[1, 5] = 1.0
    logits[2, 100] = -1.0
    inds, scores = vm.ops.moe_route(logits, 8)
    assert scores.dtype == torch.bfloat16
    assert inds[0].tolist() == list(range(8))
    assert inds[1].tolist() == [5, 0, 1, 2, 3, 4, 6, 7]
    p = torch.softmax(logits.float(), -1)
    ref = torch.gather(p, 1, inds.long()).bfloat16()
    assert torch.equal(scores, ref)


@pytest.mark.parametrize("T,k,E", [(1, 8, 128), (8, 8, 128), (32, 8, 128), (256, 8, 128), (300, 8, 128),
                                   (129, 8, 4), (700, 3, 1000)])
def test_moe_sort_bit_exact(vm, orc, cuda, T, k, E):
    """gatherSort: the stable argsort order, sorted ids and inverse order, exactly."""
    rng = np.random.default_rng(T + k + E)
    idx = rng.integers(0, E, (T, k)).astype(np.int64)
    if T == 129:
        idx[:] = 2  # one expert takes every pair: order must stay the input order
    s_ids, lhs, inv = vm.ops.moe_sort(torch.from_numpy(idx).to(cuda), E)
    order, ref_sorted, ref_inv = orc.gather_sort(idx)
    assert np.array_equal(s_ids.cpu().numpy(), ref_sorted)
    assert np.array_equal(lhs.cpu().numpy(), order // k)
    assert np.array_equal(inv.cpu().numpy(), ref_inv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_moe_combine(vm, orc, cuda, dtype):
    T, k, D = 33, 8, 2048
    g = torch.Generator(cuda).manual_seed(5)
    y = torch.randn(T * k, D, device=cuda, generator=g).bfloat16()
    sc = torch.rand(T, k, device=cuda, generator=g).to(dtype)
    perm = torch.randperm(T * k, device=cuda, generator=g).to(torch.int32)
    out = vm.ops.moe_combine(y, sc, perm)
    yy = y[perm.long()].float().reshape(T, k, D)
    prod = yy * sc.float()[:, :, None]
    if dtype == torch.bfloat16:
        prod = prod.bfloat16().float()
    ref = prod.sum(1).bfloat16()
    assert (out.float() - ref.float()).abs().max().item() <= 2 ** -7 * ref.float().abs().max().item()
    # unsorted layout, and the exact unsort (weights of one)
    out2 = vm.ops.moe_combine(y.reshape(T, k, D), sc)
    ref2 = (y.float().reshape(T, k, D) * sc.float()[:, :, None])
    ref2 = (ref2.bfloat16().float() if dtype == torch.bfloat16 else ref2).sum(1).bfloat16()
    assert (out2.float() - ref2.float()).abs().max().item() <= 2 ** -7 * ref2.float().abs().max().item()
    un = vm.scatter_unsort(y.reshape(T * k, 1, D), perm)
    assert torch.equal(un.reshape(T * k, D), y[perm.long()])


def _moe_weights(orc, vm, cuda, E, D, F):
    _, gate = make_weights(orc, vm, cuda, F, D, 64, 4, 71, lead=(E,))
    _, up = make_weights(orc, vm, cuda, F, D, 64, 4, 72, lead=(E,))
    _, down = make_weights(orc, vm, cuda, D, F, 64, 4, 73, lead=(E,))
    return gate, up, down


@pytest.mark.parametrize("T", [1, 32, 256])
def test_moe_block_config4_128_experts(vm, orc, cuda, T):
    """BASELINE config 4 at full width: 128 experts, hidden 2048, FFN 768, top-8 from
    softmax of N(0,1) fp32 logits.  Per-slot SwitchGLU outputs and the block output
    (device routing + sort + SwitchGLU + combine) against the fp64 oracle."""
    E, D, F, k = 128, 2048, 768, 8
    gate, up, down = _moe_weights(orc, vm, cuda, E, D, F)
    rng = np.random.default_rng(74 + T)
    logits = rng.normal(0, 1, (T, E)).astype(np.float32)
    xb = orc.f32_to_bf16(rng.normal(0, 1, (T, D)).astype(np.float32))
    glu = vm.SwitchGLU(vm.QuantizedSwitchLinear(*gate), vm.QuantizedSwitchLinear(*up),
                       vm.QuantizedSwitchLinear(*down))
    block = vm.switch_layers.Qwen3MoESparseMoeBlock(None, glu, k)
    x = to_dev_bf16(orc, xb, cuda)
    lg = torch.from_numpy(logits).to(cuda)
    inds, scores = block.route(lg)
    hostw = lambda t: (u32(t[0]), bits_of(t[1]), bits_of(t[2]))  # noqa: E731
    ref_slots = orc.switch_glu(xb, hostw(gate), hostw(up), hostw(down), inds.cpu().numpy().astype(np.int64))
    y = glu(x, inds)
    assert y.shape == (T, k, D)
    check_close(y.float().cpu().numpy(), ref_slots)
    out = block(x, lg)
    ref = (orc.round_bf16(ref_slots.astype(np.float32)).astype(np.float64) *
           scores.cpu().numpy().astype(np.float64)[:, :, None]).sum(1)
    assert out.shape == (T, D)
    check_close(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("case", ["sorted_lhs", "many_rows", "out_of_range"])
def test_sorted_gather_tensor_core(vm, orc, cuda, case):
    """Sorted gather_qmm with a workspace runs the expert-segmented tcgen05 GEMM
    (affine_gather_qmm_rhs semantics: bf16 weights): experts with > 64 rows (several
    tiles), x rows through lhs_indices, and ids >= n_experts (rows left zero)."""
    E, N, K = 16, 320, 512
    _, (wq, s, b) = make_weights(orc, vm, cuda, N, K, 64, 4, 91, lead=(E,))
    rng = np.random.default_rng(92)
    P = 400
    rhs = np.sort(rng.integers(0, E, P)).astype(np.int64)
    if case == "many_rows":
        rhs = np.sort(np.concatenate([np.full(150, 3), rng.integers(0, E, P - 150)])).astype(np.int64)
    if case == "out_of_range":
        rhs[-5:] = E + 2
    xb = orc.f32_to_bf16(rng.normal(0, 1, (P, 1, K)).astype(np.float32))
    lhs = rng.permutation(P).astype(np.int64) if case == "sorted_lhs" else None
    ws = torch.empty(vm.ops.gather_qmm_workspace_size(P, 1, K, E), dtype=torch.uint8, device=cuda)
    x = to_dev_bf16(orc, xb, cuda)
    li = torch.from_numpy(lhs).to(cuda) if lhs is not None else None
    ri = torch.from_numpy(rhs).to(cuda)
    y = vm.gather_quantized_mm(x, wq, s, b, lhs_indices=li, rhs_indices=ri, sorted_indices=True, workspace=ws)
    ref = orc.gather_qmm_f64(xb, u32(wq), bits_of(s), bits_of(b), lhs, rhs, 64, 4, bf16w=True)
    check_close(y.float().cpu().numpy(), ref)
    if case == "out_of_range":
        assert torch.count_nonzero(y[-5:]) == 0
