"""Loader upload: one MoE layer's packed tensors from a qmoe-rs safetensors
file into a device-resident QMoELayer (qmoe-rs src/loader.rs:204-359), and
the decoder layers' MoE blocks of a whole file as a chain
(src/loader.rs:373-459 builds the model from the same keys).

Key layout (the one quantize.py writes and src/loader.rs reads):
  layers.{l}.moe.gate.weight                          [E, H] router, f32
  layers.{l}.moe.experts.{e}.{gate,up,down}_proj.weight   packed u8 [out, in/4]
  layers.{l}.moe.experts.{e}.{gate,up,down}_proj.scales   f32 [out]
  layers.{l}.moe.shared_experts.{gate,up,down}_proj.*     optional shared FFN
  layers.{l}.moe.{gate,up,down}_proj.*                    "flattened" layer
Rules kept from the reference:
  * routed expert shapes come from the config: gate/up (I, H), down (H, I)
    (src/loader.rs:235-250); shared and flattened shapes from the stored
    tensors, in_features = 4 x the stored bytes per row (:283-300, :338-355);
  * the per-expert format is recognised by experts.0.gate_proj.weight
    (:362-365), the shared expert by shared_experts.gate_proj.weight
    (:316-318);
  * a layer without a router weight gets a uniform one, ones [E, H]
    (:410-424);
  * a missing tensor is an error naming its key (:221-232);
  * a flattened layer becomes a layer without routed experts whose FFN is
    the shared expert (:262-305, :452-456).
Tensors are read on the host (only this layer's keys) and handed to
qmoe_layer_create, which uploads them once into the stacked device layout.

Model-level helpers (the MoE part of what the reference's model loader
reads):
  * moe_config_from_tensors -- deduce_config (src/loader.rs:77-184): experts
    and hidden size from a router weight's shape, the expert width from a
    per-expert gate_proj's packed shape, top_k 6, layers = last index + 1;
  * moe_config_from_json -- parse_config_json (:186-201) with its defaults;
  * read_norm / load_block / load_block_chain -- the decoder layer's
    post_attention_layernorm (src/model.rs:366-367: eps 1e-6, weight and bias
    from layers.{l}.post_attention_layernorm, ones and zeros when the file has
    none, which is what the reference's VarBuilder creates) set on each
    layer, and the layers chained as forward_next's loop (src/model.rs:481-489).
"""
from __future__ import annotations

import dataclasses
import json
from typing import List, NamedTuple, Optional, Sequence, Tuple

import torch
from safetensors import safe_open

from .layer import BlockChain, Context, MoEConfig, QMoELayer

_PROJS = ("gate_proj", "up_proj", "down_proj")


class LayerTensors(NamedTuple):
    config: MoEConfig                    # shared_intermediate_dim from the file
    gate_weight: torch.Tensor            # [E, H] f32
    experts: List[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]]   # E x (gate, up, down)
    shared: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]]
    flattened: bool                      # no routed experts: the layer is one dense FFN


def moe_prefix(layer_idx: int) -> str:
    return f"layers.{layer_idx}.moe"


def _get(f, names, key: str, what: str) -> torch.Tensor:
    if key not in names:
        raise KeyError(f"Missing {what}: {key}")
    return f.get_tensor(key)


def _packed(f, names, base: str, what: str, shape=None):
    """(packed u8 [out, in/4], scales f32 [out]) of one projection; shape
    (out, in) checked when given, else taken from the stored bytes."""
    w = _get(f, names, base + ".weight", what + " weight")
    s = _get(f, names, base + ".scales", what + " scales")
    if w.dtype != torch.uint8 or w.dim() != 2:
        raise ValueError(f"{base}.weight: expected packed uint8 [out, in/4], got {w.dtype} {tuple(w.shape)}")
    out_f, in_f = (w.shape[0], w.shape[1] * 4) if shape is None else shape
    if tuple(w.shape) != (out_f, in_f // 4):
        raise ValueError(f"{base}.weight: shape {tuple(w.shape)}, expected ({out_f}, {in_f // 4})")
    s = s.to(torch.float32).reshape(-1)
    if s.numel() != out_f:
        raise ValueError(f"{base}.scales: {s.numel()} scales for {out_f} rows")
    return w.contiguous(), s.contiguous()


def read_layer(path: str, layer_idx: int, config: MoEConfig) -> LayerTensors:
    """Layer `layer_idx`'s router, experts and shared FFN from `path`."""
    pre = moe_prefix(layer_idx)
    E, H, I = config.num_experts, config.hidden_dim, config.intermediate_dim
    with safe_open(path, framework="pt", device="cpu") as f:
        names = set(f.keys())
        gkey = pre + ".gate.weight"
        gate = (f.get_tensor(gkey).to(torch.float32).contiguous() if gkey in names
                else torch.ones(E, H, dtype=torch.float32))
        if tuple(gate.shape) != (E, H):
            raise ValueError(f"{gkey}: shape {tuple(gate.shape)}, expected ({E}, {H})")
        experts = []
        flattened = f"{pre}.experts.0.gate_proj.weight" not in names
        if not flattened:
            for e in range(E):
                shapes = ((I, H), (I, H), (H, I))
                experts.append(tuple(
                    _packed(f, names, f"{pre}.experts.{e}.{proj}", f"expert {proj.split('_')[0]}", shp)
                    for proj, shp in zip(_PROJS, shapes)))
        base = f"{pre}.{'' if flattened else 'shared_experts.'}"
        shared = None
        if base + "gate_proj.weight" in names:
            kind = "flattened" if flattened else "shared"
            shared = tuple(_packed(f, names, base + proj, f"{kind} {proj.split('_')[0]}")
                           for proj in _PROJS)
        elif flattened:
            raise KeyError(f"Missing flattened gate weight: {base}gate_proj.weight")
    if shared is not None:
        (g, _), (u, _), (d, _) = shared
        Is = g.shape[0]
        if u.shape[0] != Is or g.shape[1] * 4 != H or u.shape[1] * 4 != H or \
                d.shape[0] != H or d.shape[1] * 4 != Is:
            raise ValueError(f"{base}*: shapes {tuple(g.shape)}, {tuple(u.shape)}, {tuple(d.shape)} "
                             f"do not form an FFN of hidden {H}")
        config = dataclasses.replace(config, shared_intermediate_dim=Is)
    else:
        config = dataclasses.replace(config, shared_intermediate_dim=0)
    return LayerTensors(config, gate, experts, shared, flattened)


def load_moe_layer(path: str, layer_idx: int, config: MoEConfig,
                   ctx: Optional[Context] = None) -> QMoELayer:
    """QMoELayer for layer `layer_idx` of `path`, weights uploaded to the
    context's device (the drop-in for the per-layer loop of src/loader.rs:430-459)."""
    t = read_layer(path, layer_idx, config)
    if t.flattened:
        # src/loader.rs:452-456: no routed experts, the dense FFN as the
        # shared expert; the layer's forward is that FFN alone
        return QMoELayer(t.config, None, [], shared=t.shared, ctx=ctx)
    return QMoELayer(t.config, t.gate_weight, t.experts, shared=t.shared, ctx=ctx)


# ---------------------------------------------------------------------------
# model-level: configuration, post-attention LayerNorm, block chains
# ---------------------------------------------------------------------------

def layer_count(path: str) -> int:
    """Layers of a file: the largest `layers.{l}.` index + 1 (src/loader.rs:95-106)."""
    last = -1
    with safe_open(path, framework="pt", device="cpu") as f:
        for name in f.keys():
            if name.startswith("layers."):
                idx = name.split(".")[1]
                if idx.isdigit():
                    last = max(last, int(idx))
    return last + 1


def moe_config_from_tensors(path: str) -> MoEConfig:
    """The MoE configuration deduce_config (src/loader.rs:77-184) reads from
    tensor shapes: num_experts and hidden_dim from a `moe.gate.weight`, then
    intermediate_dim and hidden_dim (4 x the packed bytes per row) from a
    per-expert `gate_proj.weight`; top_k is 6.  Where the reference takes the
    first matching name of the file's unordered key list, the per-expert
    projections of the lowest layer are used (a flattened layer's
    `moe.gate_proj.weight` is not an expert's)."""
    E = H = I = None
    with safe_open(path, framework="pt", device="cpu") as f:
        names = sorted(f.keys())
        for n in names:
            if n.endswith("moe.gate.weight"):
                shp = f.get_slice(n).get_shape()
                if len(shp) == 2:
                    E, H = int(shp[0]), int(shp[1])
                    break
        experts = [n for n in names if ".moe.experts." in n and n.endswith(".gate_proj.weight")]
        if experts:
            shp = f.get_slice(experts[0]).get_shape()
            if len(shp) == 2:
                I, H = int(shp[0]), 4 * int(shp[1])
    if E is None or H is None or I is None:
        raise KeyError("the file has no router weight or no per-expert gate_proj to deduce the "
                       "MoE configuration from")
    return MoEConfig(E, 6, H, I)


def moe_config_from_json(path: str) -> Tuple[MoEConfig, int]:
    """(MoE configuration, layers) from a config.json as parse_config_json
    (src/loader.rs:186-201) reads it, with its defaults: hidden_size 2048,
    num_layers | num_hidden_layers 27, num_experts | num_local_experts 64,
    top_k | num_experts_per_tok 6, intermediate_dim | intermediate_size 1408,
    hidden_dim = hidden_size."""
    with open(path) as fh:
        c = json.load(fh)

    def first(*keys, default):
        for k in keys:
            if c.get(k) is not None:
                return c[k]
        return default

    hidden = int(first("hidden_size", default=2048))
    cfg = MoEConfig(int(first("num_experts", "num_local_experts", default=64)),
                    int(first("top_k", "num_experts_per_tok", default=6)),
                    int(first("hidden_dim", default=hidden)),
                    int(first("intermediate_dim", "intermediate_size", default=1408)))
    return cfg, int(first("num_layers", "num_hidden_layers", default=27))


def read_norm(path: str, layer_idx: int, hidden: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(weight, bias) [hidden] f32 of layer `layer_idx`'s post_attention_layernorm;
    ones and zeros when the file has none (the values the reference's
    VarBuilder gives a LayerNorm missing from the file)."""
    pre = f"layers.{layer_idx}.post_attention_layernorm"
    with safe_open(path, framework="pt", device="cpu") as f:
        names = set(f.keys())
        w = (f.get_tensor(pre + ".weight").to(torch.float32).reshape(-1) if pre + ".weight" in names
             else torch.ones(hidden, dtype=torch.float32))
        b = (f.get_tensor(pre + ".bias").to(torch.float32).reshape(-1) if pre + ".bias" in names
             else torch.zeros(hidden, dtype=torch.float32))
    for t, k in ((w, "weight"), (b, "bias")):
        if t.numel() != hidden:
            raise ValueError(f"{pre}.{k}: {t.numel()} values for hidden size {hidden}")
    return w.contiguous(), b.contiguous()


NORM_EPS = 1e-6        # candle_nn::layer_norm(hidden, 1e-6, ...) (src/model.rs:367)


def load_block(path: str, layer_idx: int, config: MoEConfig,
               ctx: Optional[Context] = None) -> QMoELayer:
    """Layer `layer_idx`'s MoE block: the MoE layer with its post-attention
    LayerNorm set, ready for forward_block (src/model.rs:400-412)."""
    layer = load_moe_layer(path, layer_idx, config, ctx=ctx)
    w, b = read_norm(path, layer_idx, config.hidden_dim)
    layer.set_norm(w, b, NORM_EPS)
    return layer


def load_block_chain(path: str, config: MoEConfig, layers: Optional[Sequence[int]] = None,
                     ctx: Optional[Context] = None) -> BlockChain:
    """The MoE blocks of `layers` (default: every layer of the file, in
    order) chained as forward_next's layer loop (src/model.rs:481-489);
    flattened layers take part as their FFN."""
    idx = list(layers) if layers is not None else list(range(layer_count(path)))
    if not idx:
        raise ValueError("no layers to chain")
    return BlockChain([load_block(path, l, config, ctx=ctx) for l in idx])
