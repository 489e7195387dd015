"""Shared helpers of the test suite: seeded synthetic layers and tolerances."""
from __future__ import annotations

import numpy as np
import torch

from qmoe_b200 import quantize as qz


def rel_err(a, b) -> float:
    """max |a - b| / max |b| (the max-abs relative error of the parity bar)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = max(float(np.max(np.abs(b))) if b.size else 0.0, 1e-30)
    return float(np.max(np.abs(a - b))) / den if a.size else 0.0


def synth_layer(E, H, I, Is=0, seed=1234, device="cpu", std=0.02):
    """Seeded N(0, std) expert weights packed by the qmoe-rs format producer,
    an f32 N(0, 0.02) gate.  Returns torch tensors on `device`:
    (experts [E][(gate), (up), (down)] of (packed, scales), shared or None,
    gate_w [E, H])."""
    g = torch.Generator(device=device).manual_seed(seed)

    def mat(o, i):
        w = torch.randn(o, i, generator=g, device=device) * std
        return qz.quantize_weight(w)

    experts = [[mat(I, H), mat(I, H), mat(H, I)] for _ in range(E)]
    shared = [mat(Is, H), mat(Is, H), mat(H, Is)] if Is else None
    gate_w = torch.randn(E, H, generator=g, device=device) * 0.02
    return experts, shared, gate_w


def to_numpy_experts(experts):
    return [[(p.cpu().numpy().reshape(-1), s.cpu().numpy()) for p, s in ex]
            for ex in experts]
