"""GPU parity of the MXFP4 path (csrc/fpquant.cu) against the numpy restatement of MLX's
fp_quantize / fp_dequantize / fp qdot (oracle.mxfp4_*), through the C ABI.

Bars: e2m1 codes and e8m0 scale bytes bit-exact (bf16 and f32 inputs, with zero groups, values
on the e2m1 grid and on its midpoints); dequantized values bit-exact (f32 exact, bf16 rounded
once); the matmul within the GEMV tolerance (max 1e-2 / mean 1e-3 relative to the fp64 oracle)."""
import numpy as np
import pytest
import torch

from test_quant_gpu import bits_of, check_close, to_dev_bf16, u32

pytestmark = pytest.mark.gpu


def _weights(orc, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    w[0, :32] = 0.0                                                      # an all-zero group
    w[1, :32] = np.array([6, -3, 0.5, 0.25, 0.75, 1.25, 2.5, 5] * 4)      # grid values and midpoints
    w[2, 32:64] = np.linspace(-1e-3, 1e-3, 32)
    return w


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_mxfp4_quantize_dequantize_bit_exact(vm, orc, cuda, dtype):
    w = _weights(orc, 64, 512, 1)
    if dtype == "bf16":
        wb = orc.f32_to_bf16(w)
        wt = to_dev_bf16(orc, wb, cuda)
        w = orc.bf16_to_f32(wb)
    else:
        wt = torch.from_numpy(w).to(cuda)
    wq, sc = vm.ops.fp_quantized(wt)
    rq, rs = orc.mxfp4_quantize(w)
    assert np.array_equal(u32(wq), rq)
    assert np.array_equal(sc.cpu().numpy(), rs)
    vals = orc.mxfp4_values(rq, rs)
    f32 = vm.ops.fp_dequantized(wq, sc, dtype=torch.float32).cpu().numpy()
    assert np.array_equal(f32, vals)
    b16 = vm.ops.fp_dequantized(wq, sc, dtype=torch.bfloat16)
    assert np.array_equal(bits_of(b16), orc.f32_to_bf16(vals))


@pytest.mark.parametrize("M", [1, 3, 8, 33])
@pytest.mark.parametrize("N,K", [(272, 1024), (4096, 4096)])
def test_mxfp4_matmul(vm, orc, cuda, M, N, K):
    w = _weights(orc, N, K, 2 + M)
    wq, sc = vm.ops.fp_quantized(torch.from_numpy(w).to(cuda))
    rng = np.random.default_rng(M)
    xb = orc.f32_to_bf16(rng.normal(0, 1, (M, K)).astype(np.float32))
    y = vm.ops.fp_quantized_mm(to_dev_bf16(orc, xb, cuda), wq, sc)
    rows = np.arange(0, N, 7)
    ref = orc.mxfp4_qmm_f64(xb, u32(wq)[rows], sc.cpu().numpy()[rows])
    check_close(y.float().cpu().numpy()[:, rows], ref)


def test_mxfp4_rejects_other_modes(vm, cuda):
    w = torch.randn(8, 64, device=cuda).bfloat16()
    with pytest.raises(vm.VMLXError):
        vm.ops.fp_quantized(w, group_size=64)
    with pytest.raises(vm.VMLXError):
        vm.ops.fp_quantized(w, mode="nvfp4")


def test_mxfp4_quantized_linear_and_loader(vm, cuda, tmp_path):
    """QuantizedLinear in mode mxfp4, and the same layer through a written-and-read checkpoint."""
    import json
    g = torch.Generator(cuda).manual_seed(5)
    w = (torch.randn(256, 512, device=cuda, generator=g) * 0.02).bfloat16()
    ql = vm.QuantizedLinear.from_weight(w, group_size=32, bits=4, mode="mxfp4")
    x = torch.randn(2, 512, device=cuda, generator=g).bfloat16()
    assert torch.equal(ql(x), vm.ops.fp_quantized_mm(x, ql.weight, ql.scales))
    vm.load.write_safetensors(str(tmp_path / "m.safetensors"), {"model.proj.weight": ql.weight,
                                                                "model.proj.scales": ql.scales},
                              u32=["model.proj.weight"])
    json.dump({"quantization": {"group_size": 32, "bits": 4, "mode": "mxfp4"}}, open(tmp_path / "config.json", "w"))
    mods, _, _ = vm.load.load_quantized_model(str(tmp_path), ["proj"], device=cuda)
    assert mods["proj"].mode == "mxfp4" and torch.equal(mods["proj"](x), ql(x))
