"""Loader upload: one MoE layer's packed tensors from a qmoe-rs safetensors
file into a device-resident QMoELayer (qmoe-rs src/loader.rs:204-359).

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
"""
from __future__ import annotations

import dataclasses
from typing import List, NamedTuple, Optional, Tuple

import torch
from safetensors import safe_open

from .layer import Context, MoEConfig, QMoELayer

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
