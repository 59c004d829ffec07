"""Pre-quantized checkpoint loading (vmlx-swift_b200/load.py), after the reference's
BaseConfiguration quantization block and Load.swift's quantized-module construction.

CPU: the config parser (default, per-layer dicts, `false` skips, scalar metadata ignored,
an override without group_size takes the default's), path resolution across `model.` /
`language_model.` spellings and `attn` / `self_attn`, a safetensors round trip, layer
construction from `.weight` / `.scales` / `.biases` (bits and group size per layer, skips,
width mismatch rejected, MXFP stamp over an affine payload loaded as affine).
GPU: a layer built from a written-and-read checkpoint computes the same bits as the layer
built from the in-memory tensors."""
import json
import os

import numpy as np
import pytest
import torch

CONFIG = {"model_type": "llama", "quantization": {
    "group_size": 64, "bits": 4, "quant_method": "mlx", "lm_head_bits": 8, "attention_bits": [4, 8],
    "model.layers.0.mlp.down_proj": {"group_size": 32, "bits": 8},
    "model.layers.0.self_attn.o_proj": {"bits": 8},
    "lm_head": False}}


def _q(n, k, gs, bits, seed):
    """Random packed codes / scales / biases of an [n, k] affine-quantized matrix (CPU)."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-(1 << 31), 1 << 31, (n, k * bits // 32), generator=g, dtype=torch.int32)
    s = (torch.rand(n, k // gs, generator=g) * 0.01).bfloat16()
    b = (-torch.rand(n, k // gs, generator=g) * 0.05).bfloat16()
    return w, s, b


def test_parse_quantization(vm):
    plq = vm.load.parse_quantization(CONFIG)
    Q = vm.load.Quantization
    assert plq.quantization("model.layers.3.mlp.up_proj") == Q(64, 4)
    assert plq.quantization("model.layers.0.mlp.down_proj") == Q(32, 8)
    assert plq.quantization("layers.0.mlp.down_proj") == Q(32, 8)           # module path without `model.`
    assert plq.quantization("language_model.model.layers.0.mlp.down_proj") == Q(32, 8)
    assert plq.quantization("model.layers.0.attn.o_proj") == Q(64, 8)       # attn alias, default group size
    assert plq.quantization("lm_head") is None                              # `false`: not quantized
    assert set(plq.per_layer) == {"model.layers.0.mlp.down_proj", "model.layers.0.self_attn.o_proj", "lm_head"}
    assert vm.load.parse_quantization({"model_type": "llama"}) is None


def test_safetensors_round_trip_and_modules(vm, tmp_path):
    tensors = {}
    for name, (n, k, gs, bits) in {"model.layers.0.mlp.down_proj": (64, 256, 32, 8),
                                   "model.layers.0.mlp.up_proj": (256, 64, 64, 4),
                                   "model.layers.0.self_attn.o_proj": (64, 128, 64, 8),
                                   "lm_head": (100, 64, 64, 4),
                                   "model.embed_tokens": (100, 64, 64, 4)}.items():
        w, s, b = _q(n, k, gs, bits, len(tensors))
        tensors[f"{name}.weight"], tensors[f"{name}.scales"], tensors[f"{name}.biases"] = w, s, b
    tensors["model.norm.weight"] = torch.ones(64).bfloat16()
    # an expert stack (SwitchLinear)
    we = torch.stack([_q(32, 64, 64, 4, 10 + e)[0] for e in range(4)])
    tensors["model.layers.0.mlp.switch_mlp.gate_proj.weight"] = we
    tensors["model.layers.0.mlp.switch_mlp.gate_proj.scales"] = torch.ones(4, 32, 1).bfloat16()
    tensors["model.layers.0.mlp.switch_mlp.gate_proj.biases"] = torch.zeros(4, 32, 1).bfloat16()
    u32 = [k for k in tensors if k.endswith(".weight") and tensors[k].dtype == torch.int32]
    vm.load.write_safetensors(str(tmp_path / "model.safetensors"), tensors, u32=u32)
    json.dump(CONFIG, open(tmp_path / "config.json", "w"))
    back = vm.load.read_safetensors(str(tmp_path / "model.safetensors"))
    assert set(back) == set(tensors)
    for k, t in tensors.items():
        assert back[k].dtype == t.dtype and torch.equal(back[k].view(torch.int16) if t.dtype == torch.bfloat16
                                                        else back[k], t.view(torch.int16)
                                                        if t.dtype == torch.bfloat16 else t), k
    paths = ["layers.0.mlp.down_proj", "layers.0.mlp.up_proj", "layers.0.self_attn.o_proj", "lm_head",
             "embed_tokens", "layers.0.mlp.switch_mlp.gate_proj", "layers.0.mlp.gate_proj"]
    mods, plq, rest = vm.load.load_quantized_model(str(tmp_path), paths)
    assert set(mods) == {"layers.0.mlp.down_proj", "layers.0.mlp.up_proj", "layers.0.self_attn.o_proj",
                         "embed_tokens", "layers.0.mlp.switch_mlp.gate_proj"}   # lm_head skipped, gate absent
    d = mods["layers.0.mlp.down_proj"]
    assert (d.group_size, d.bits) == (32, 8) and d.shape == (64, 256)
    assert (mods["layers.0.self_attn.o_proj"].bits, mods["layers.0.self_attn.o_proj"].group_size) == (8, 64)
    assert mods["layers.0.mlp.switch_mlp.gate_proj"].num_experts == 4
    assert mods["embed_tokens"][3:] == (64, 4)
    assert "lm_head.weight" in rest and "model.norm.weight" in rest and "model.layers.0.mlp.up_proj.weight" not in rest


def test_width_mismatch_and_mxfp_fallback(vm):
    w, s, b = _q(16, 128, 64, 4, 1)
    weights = {"model.x.weight": w, "model.x.scales": s, "model.x.biases": b}
    bad = vm.load.PerLayerQuantization(vm.load.Quantization(64, 8), {})
    with pytest.raises(vm.VMLXError):
        vm.load.quantized_modules(weights, ["x"], bad)
    mx = vm.load.PerLayerQuantization(vm.load.Quantization(64, 4, "mxfp4"), {})
    m = vm.load.quantized_modules(weights, ["x"], mx)["x"]
    assert m.mode == "affine" and m.bits == 4


@pytest.mark.gpu
def test_loaded_layer_matches_direct(vm, cuda, tmp_path):
    g = torch.Generator(cuda).manual_seed(0)
    w = (torch.randn(512, 1024, device=cuda, generator=g) * 0.02).bfloat16()
    direct = vm.QuantizedLinear.from_weight(w, group_size=64, bits=4)
    vm.load.write_safetensors(str(tmp_path / "m.safetensors"),
                              {"model.layers.0.mlp.up_proj.weight": direct.weight,
                               "model.layers.0.mlp.up_proj.scales": direct.scales,
                               "model.layers.0.mlp.up_proj.biases": direct.biases},
                              u32=["model.layers.0.mlp.up_proj.weight"])
    json.dump({"quantization": {"group_size": 64, "bits": 4}}, open(tmp_path / "config.json", "w"))
    mods, _, _ = vm.load.load_quantized_model(str(tmp_path), ["layers.0.mlp.up_proj"], device=cuda)
    x = torch.randn(3, 1024, device=cuda, generator=g).bfloat16()
    assert torch.equal(mods["layers.0.mlp.up_proj"](x), direct(x))
