"""CPU tests of the oracle: known-answer fixtures of the reference's own tests,
edge cases of the quantize rule, and a second, vectorised numpy restatement
of affine_quantize (quantized.h:2393-2496) checked bit for bit against the C
restatement."""
import numpy as np
import pytest


def np_quantize(w32: np.ndarray, gs: int, bits: int):
    """Independent numpy restatement of affine_quantize in fp32 (codes + fp32 scale/bias)."""
    w = w32.astype(np.float32).reshape(-1, gs)
    n_bins = np.float32((1 << bits) - 1)
    w_min = np.minimum(w.min(1), np.float32(np.finfo(np.float32).max))
    w_max = np.maximum(w.max(1), np.float32(0))
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7)).astype(np.float32)
        side = np.abs(w_min) > np.abs(w_max)
        scale = np.where(side, scale, -scale).astype(np.float32)
        edge = np.where(side, w_min, w_max).astype(np.float32)
        q0 = np.trunc(edge / scale + np.copysign(np.float32(0.5), edge / scale)).astype(np.float32)
        # roundf is half away from zero; guard against x.5 representation issues
        r = edge / scale
        q0 = np.where(np.abs(r - np.trunc(r)) == 0.5, np.trunc(r) + np.sign(r), np.round(r)).astype(np.float32)
        at_zero = q0 == 0
        scale = np.where(at_zero, scale, edge / q0).astype(np.float32)
        bias = np.where(at_zero, np.float32(0), edge).astype(np.float32)
        v = (w - bias[:, None]) / scale[:, None]
    q = np.where(np.abs(v - np.trunc(v)) == 0.5, np.trunc(v) + np.sign(v), np.round(v))
    q = np.minimum(q, n_bins)
    q = np.where(q > 0, q, 0).astype(np.uint32)
    return q, scale, bias


def pack(q: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    q = q.reshape(q.shape[0], -1, per).astype(np.uint32)
    sh = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(q << sh, axis=2)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_c_oracle_matches_numpy_restatement(orc, bits, gs):
    rng = np.random.default_rng(1000 + bits * 7 + gs)
    rows, K = 24, 4 * gs
    w = rng.normal(0, 0.02, (rows, K)).astype(np.float32)
    w[0, :gs] = -np.abs(w[0, :gs])          # all-negative group: w_max stays 0
    w[1, :gs] = 0.0                          # all-zero group
    w[2, :gs] = 0.25                         # constant positive group
    wq, s, b = orc.quantize(w, gs, bits, dtype="f32")
    q, s_np, b_np = np_quantize(w, gs, bits)
    assert np.array_equal(s.reshape(-1).view(np.uint32), s_np.view(np.uint32))
    assert np.array_equal(b.reshape(-1).view(np.uint32), b_np.view(np.uint32))
    assert np.array_equal(wq, pack(q.reshape(rows, K), bits).reshape(rows, -1))


def test_quantize_shapes_opstests(orc):
    """Tests/MLXTests/OpsTests.swift:96-115: quantized([8,64]) -> wq [8,8] u32, scales/biases [8,1]."""
    a = np.random.default_rng(0).uniform(0, 1, (8, 64)).astype(np.float32)
    wq, s, b = orc.quantize(a, 64, 4, dtype="f32")
    assert wq.shape == (8, 8) and wq.dtype == np.uint32
    assert s.shape == (8, 1) and b.shape == (8, 1)


def test_known_answer_gather_qmm_fixture(orc):
    """Tests/MLXTests/QuantizationTests.swift:65-111: arange fixture, gs 32, b4,
    gather_qmm over rhsIndices [0, 2] equals dequantized + matmul (rtol=atol=1e-3).
    The fixture values are exact in bf16, so the bf16 path is checked too."""
    dense = (np.arange(3 * 16 * 32, dtype=np.float32).reshape(3, 16, 32) / 2048) - 0.5
    x = (np.arange(2 * 1 * 32, dtype=np.float32).reshape(2, 1, 32) / 128) - 0.25
    rhs = np.array([0, 2])
    # float32 path, as the reference test runs it
    wq, s, b = orc.quantize(dense, 32, 4, dtype="f32")
    assert wq.shape == (3, 16, 4) and s.shape == (3, 16, 1)
    deq = orc.dequantize(wq, s, b, 32, 4)
    expected = np.concatenate([x[0] @ deq[0].T, x[1] @ deq[2].T], 0)
    got = np.concatenate([x[i] @ deq[rhs[i]].T for i in range(2)], 0)
    np.testing.assert_allclose(got, expected, rtol=1e-3, atol=1e-3)
    assert np.all(np.abs(deq - dense) <= np.abs(s) + 1e-7)
    # bf16 path: x is exact in bf16; the gathered oracle matmul must equal
    # dequantized + matmul of the same bf16-quantized weights
    assert np.array_equal(orc.round_bf16(x), x)
    wqb, sb, bb = orc.quantize(dense, 32, 4, dtype="bf16")
    deqb = orc.dequantize(wqb, sb, bb, 32, 4)
    expb = np.concatenate([x[i].astype(np.float64) @ deqb[rhs[i]].T.astype(np.float64) for i in range(2)], 0)
    gotb = orc.gather_qmm_f64(orc.f32_to_bf16(x), wqb, sb, bb, None, rhs, 32, 4)
    np.testing.assert_allclose(gotb.reshape(2, 16), expb, rtol=1e-3, atol=1e-3)


def test_dequantize_error_bound(orc):
    """Round-trip error stays within one quantization step.  (Not half a step:
    the edge rule snaps the grid to the larger-magnitude extreme and shrinks the
    step to edge/q0, so values at the far end can clip at 2^bits-1.)"""
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (64, 512)).astype(np.float32)
    for bits in (4, 8):
        wq, s, b = orc.quantize(w, 64, bits, dtype="f32")
        deq = orc.dequantize(wq, s, b, 64, bits)
        step = np.abs(s).repeat(64, axis=1)
        assert np.all(np.abs(deq - w) <= step * (1 + 1e-5) + 1e-7)


def test_qmm_fp32_agrees_with_f64(orc):
    rng = np.random.default_rng(4)
    w = rng.normal(0, 0.02, (128, 1024)).astype(np.float32)
    x = orc.f32_to_bf16(rng.normal(0, 1, (3, 1024)).astype(np.float32))
    wq, s, b = orc.quantize(w, 64, 4)
    y64 = orc.qmm_f64(x, wq, s, b, 64, 4)
    y32 = orc.bf16_to_f32(orc.qmm_fp32_bf16(x, wq, s, b, 64, 4))
    np.testing.assert_allclose(y32, y64, rtol=1e-2, atol=1e-2 * np.abs(y64).max())


def test_gather_sort_permutations(orc):
    idx = np.array([[3, 1], [1, 0], [3, 2]], np.uint32)
    order, sidx, inv = orc.gather_sort(idx)
    assert list(sidx) == [0, 1, 1, 2, 3, 3]
    assert list(order) == [3, 1, 2, 5, 0, 4]  # stable
    assert np.array_equal(sidx[inv], idx.reshape(-1))


def test_mxfp4_oracle_known_answers(orc):
    """Hand-computed groups: max 6 -> scale 1 (e8m0 127), values on the grid map to their codes,
    midpoints go to the even mantissa (0.25 -> 0, 0.75 -> 1.0, 1.25 -> 1.0, 2.5 -> 2.0, 5 -> 4.0);
    an all-zero group gets the smallest scale (bits 0) and zero codes; max 3 -> scale 0.5 (126)."""
    import numpy as np
    g = np.array([6, -3, 0.5, 0.25, 0.75, 1.25, 2.5, 5] + [0] * 24, np.float32)
    w = np.stack([g, np.zeros(32, np.float32), g / 2]).astype(np.float32)
    wq, sc = orc.mxfp4_quantize(w)
    assert sc.ravel().tolist() == [127, 0, 126]
    codes = [(int(wq[0, 0]) >> (4 * i)) & 0xF for i in range(8)]
    assert codes == [7, 8 | 5, 1, 0, 2, 2, 4, 6]
    assert wq[1].tolist() == [0, 0, 0, 0]
    assert np.array_equal(wq[2], wq[0])  # the same codes at half the scale
    v = orc.mxfp4_values(wq, sc)
    assert v[0, :8].tolist() == [6.0, -3.0, 0.5, 0.0, 1.0, 1.0, 2.0, 4.0]
    assert v[2, 0] == 3.0
