"""Pre-quantized safetensors checkpoints onto this library's layers (row f2).

Mirrors the reference loader's quantized path:
  * the `quantization` block of config.json (Libraries/MLXLMCommon/BaseConfiguration.swift:
    225-337): the default {group_size, bits, mode}, per-layer overrides (a dict, or `false` to
    skip a layer), and the scalar / list metadata keys that are not overrides;
  * per-layer resolution with the checkpoint's path spellings (`model.` / `language_model.`
    prefixes, `attn` / `self_attn`) (BaseConfiguration.swift:86-200);
  * building QuantizedLinear / QuantizedSwitchLinear / quantized embeddings straight from the
    `.weight` (u32 codes) + `.scales` (+ `.biases`) tensors, the affine fallback when an MXFP
    bundle still carries `.biases` (Libraries/MLXLMCommon/Load.swift:740-830).
The on-disk layout is already the kernels' layout, so loading is a copy to the device.

safetensors: an 8-byte little-endian header length, a JSON header {name: {dtype, shape,
data_offsets}}, then the raw tensor bytes (the published format).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch

from ._lib import VMLXError, VMLX_E_INVALID, VMLX_E_UNSUPPORTED

_ST_DTYPES = {"U32": (np.uint32, torch.int32), "I32": (np.int32, torch.int32), "BF16": (np.uint16, torch.bfloat16),
              "F16": (np.float16, torch.float16), "F32": (np.float32, torch.float32), "U8": (np.uint8, torch.uint8),
              "I64": (np.int64, torch.int64)}
_TORCH_TO_ST = {torch.int32: "I32", torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32",
                torch.uint8: "U8", torch.int64: "I64"}
if hasattr(torch, "uint32"):
    _TORCH_TO_ST[torch.uint32] = "U32"


def read_safetensors(path: str, device=None) -> Dict[str, torch.Tensor]:
    """All tensors of one .safetensors file (U32 codes come back as int32 with the same bits)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            np_dt, t_dt = _ST_DTYPES[meta["dtype"]]
            s, e = meta["data_offsets"]
            f.seek(base + s)
            a = np.frombuffer(f.read(e - s), dtype=np_dt).reshape(meta["shape"]).copy()
            if meta["dtype"] == "U32":
                a = a.view(np.int32)
            t = torch.from_numpy(a)
            if meta["dtype"] == "BF16":
                t = t.view(torch.bfloat16)
            out[name] = t.to(device) if device is not None else t
    return out


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor], u32: Iterable[str] = ()) -> None:
    """Write tensors (names in `u32` are stored with dtype U32: packed codes)."""
    u32 = set(u32)
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        if hasattr(torch, "uint32") and t.dtype == torch.uint32:
            t = t.view(torch.int32)
        raw = t.view(torch.int16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
        dt = "U32" if name in u32 else _TORCH_TO_ST[t.dtype]
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def load_weights(model_dir: str, device=None) -> Dict[str, torch.Tensor]:
    """Every *.safetensors file of a model directory, merged."""
    out: Dict[str, torch.Tensor] = {}
    for fn in sorted(os.listdir(model_dir)):
        if fn.endswith(".safetensors"):
            out.update(read_safetensors(os.path.join(model_dir, fn), device))
    return out


@dataclass(frozen=True)
class Quantization:
    group_size: int
    bits: int
    mode: str = "affine"


SKIP = "skip"
# keys of the quantization block that are not per-layer instructions
_NON_LAYER_KEYS = {"group_size", "bits", "mode", "quant_method", "linear_class", "quantization_mode", "mxtq_bits",
                   "routed_expert_bits", "routed_expert_bit_plan", "mxtq_seed", "expert_layout", "embed_bits",
                   "router_bits", "attention_bits", "lm_head_bits", "cca_conv_bits", "norms_residual_bits"}


def _path_candidates(layer: str) -> List[str]:
    """The spellings a module path may have in checkpoint metadata, most specific first."""
    out: List[str] = []

    def add(v):
        if v not in out:
            out.append(v)

    def add_attn(v):
        add(v)
        if ".attn." in v:
            add(v.replace(".attn.", ".self_attn."))
        elif v.endswith(".attn"):
            add(v[:-len(".attn")] + ".self_attn")
        elif ".self_attn." in v:
            add(v.replace(".self_attn.", ".attn."))
        elif v.endswith(".self_attn"):
            add(v[:-len(".self_attn")] + ".attn")

    add_attn(layer)
    if layer.startswith("language_model.model."):
        mp = layer[len("language_model."):]
        add_attn(mp)
        add_attn(mp[len("model."):])
    elif layer.startswith("language_model."):
        inner = layer[len("language_model."):]
        add_attn(inner)
        add_attn(inner[len("model."):] if inner.startswith("model.") else "model." + inner)
    elif layer.startswith("model."):
        bare = layer[len("model."):]
        add_attn(bare)
        add_attn("language_model." + layer)
    else:
        add_attn("model." + layer)
        add_attn("language_model." + layer)
        add_attn("language_model.model." + layer)
    return out


class PerLayerQuantization:
    """The default quantization plus per-layer overrides (Quantization or SKIP)."""

    def __init__(self, default: Optional[Quantization], per_layer: Dict[str, object]):
        self.default, self.per_layer = default, per_layer

    def quantization(self, layer: str) -> Optional[Quantization]:
        for c in _path_candidates(layer):
            if c in self.per_layer:
                o = self.per_layer[c]
                return None if o == SKIP else o
        return self.default


def parse_quantization(config: dict) -> Optional[PerLayerQuantization]:
    """The `quantization` (or `quantization_config`) block of a config.json dict."""
    q = config.get("quantization", config.get("quantization_config"))
    if q is None:
        return None
    if "group_size" not in q or "bits" not in q:
        raise VMLXError(VMLX_E_INVALID, "quantization block without group_size / bits")
    default = Quantization(int(q["group_size"]), int(q["bits"]), str(q.get("mode", "affine")).lower())
    per: Dict[str, object] = {}
    for k, v in q.items():
        if k in _NON_LAYER_KEYS:
            continue
        if isinstance(v, bool):
            if not v:
                per[k] = SKIP
        elif isinstance(v, (str, int, float, list)):
            continue  # converter / runtime metadata, not a layer override
        elif isinstance(v, dict):
            if "bits" not in v:
                raise VMLXError(VMLX_E_INVALID, f"quantization override {k!r} without bits")
            per[k] = Quantization(int(v.get("group_size", default.group_size)), int(v["bits"]),
                                  str(v.get("mode", "affine")).lower())
    return PerLayerQuantization(default, per)


def quantized_modules(weights: Dict[str, torch.Tensor], paths: Iterable[str], plq: PerLayerQuantization):
    """{module path: layer} for every path whose `.weight` + `.scales` exist under one of its
    spellings: 2-D weights -> nn.QuantizedLinear, 3-D (experts) -> QuantizedSwitchLinear, paths
    ending in `embed_tokens` -> (w, scales, biases, group_size, bits) for the embedding kernel."""
    from .nn import QuantizedLinear
    from .switch_layers import QuantizedSwitchLinear
    out = {}
    for path in paths:
        base = next((b for b in _path_candidates(path) if f"{b}.weight" in weights and f"{b}.scales" in weights),
                    None)
        if base is None:
            continue
        q = plq.quantization(path)
        if q is None:
            continue
        mode = q.mode
        if f"{base}.biases" in weights and mode in ("mxfp4", "mxfp8"):
            mode = "affine"  # an MXFP stamp over an affine payload: load it as affine
        if mode not in ("affine", "mxfp4"):
            raise VMLXError(VMLX_E_UNSUPPORTED, f"{path}: quantization mode {mode!r} (affine, mxfp4)")
        w, s = weights[f"{base}.weight"], weights[f"{base}.scales"]
        bq = weights.get(f"{base}.biases")
        bias = weights.get(f"{base}.bias")
        if w.shape[-1] * 32 // q.bits != s.shape[-1] * q.group_size:
            raise VMLXError(VMLX_E_INVALID, f"{path}: packed width {w.shape[-1]} does not match "
                                            f"{q.bits}-bit groups of {q.group_size} ({s.shape[-1]} groups)")
        if mode == "mxfp4" and (w.dim() != 2 or path.endswith("embed_tokens")):
            raise VMLXError(VMLX_E_UNSUPPORTED, f"{path}: mxfp4 is supported for dense linears only")
        if path.endswith("embed_tokens"):
            out[path] = (w, s, bq, q.group_size, q.bits)
        elif w.dim() == 3:
            out[path] = QuantizedSwitchLinear(w, s, bq, bias, q.group_size, q.bits, mode)
        else:
            out[path] = QuantizedLinear(w, bias, s, bq, q.group_size, q.bits, mode)
    return out


def load_quantized_model(model_dir: str, paths: Iterable[str], device=None):
    """config.json + *.safetensors of a pre-quantized model directory -> ({path: layer}, the
    per-layer quantization, the remaining (unquantized) tensors)."""
    with open(os.path.join(model_dir, "config.json")) as f:
        config = json.load(f)
    plq = parse_quantization(config)
    if plq is None:
        raise VMLXError(VMLX_E_INVALID, f"{model_dir}: config.json has no quantization block")
    weights = load_weights(model_dir, device)
    mods = quantized_modules(weights, paths, plq)
    used = set()
    for path in mods:
        for b in _path_candidates(path):
            used.update(k for k in (f"{b}.weight", f"{b}.scales", f"{b}.biases", f"{b}.bias") if k in weights)
    rest = {k: v for k, v in weights.items() if k not in used}
    return mods, plq, rest
