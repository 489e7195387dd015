"""Regenerate the golden fixtures in this directory from qmoe-rs itself.

Runs only where the qmoe-rs sources are checked out (it imports the
project's own offline quantizer, quantize.py, whose quantize_and_pack and
std-scale step define the packed format).  The GPU boxes never run it; the
tests read the committed .npz files.

Usage:  python tests/golden/make_golden.py /path/to/qmoe-rs

Fixtures:
  quant_small.npz   seeded N(0, 0.02) weights [24, 64] and [16, 128]; the
                    scales and packed bytes qmoe-rs's quantize.py produces
                    (std(dim=1).clamp(min=1e-5), quantize_and_pack).
  quant_edges.npz   explicit rounding/clamp edge cases with scale 1 (ties
                    at +-0.5, +-1.5, +-2.5 round half to even; |x| > 1
                    clamps) plus an all-constant row (std 0 -> 1e-5).
  moe_tiny.npz      a tiny MoE layer (E=4, H=64, I=128, shared I_s=128)
                    whose expert weights were packed by quantize.py, with
                    a seeded gate and input; used by the CPU oracle tests
                    and the GPU parity tests.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_quantizer(ref_root: str):
    spec = importlib.util.spec_from_file_location(
        "qmoe_rs_quantize", os.path.join(ref_root, "quantize.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_pack(ref, w: torch.Tensor):
    # the exact steps of quantize.py:97-105
    scale = w.std(dim=1)
    scale = torch.clamp(scale, min=1e-5)
    packed = ref.quantize_and_pack(w, scale)
    return packed.numpy(), scale.numpy().astype(np.float32)


def main(ref_root: str):
    ref = load_reference_quantizer(ref_root)

    g = torch.Generator().manual_seed(1234)
    w_a = torch.randn(24, 64, generator=g) * 0.02
    w_b = torch.randn(16, 128, generator=g) * 0.02
    pa, sa = ref_pack(ref, w_a)
    pb, sb = ref_pack(ref, w_b)
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"),
                        w_a=w_a.numpy(), packed_a=pa, scales_a=sa,
                        w_b=w_b.numpy(), packed_b=pb, scales_b=sb)

    edges = torch.tensor([
        [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 0.49999997, -0.49999997,
         0.50000006, -0.50000006, 1.0, -1.0, 0.0, -0.0, 7.0, -7.0],
        [0.25, 0.75, -0.25, -0.75, 1e-8, -1e-8, 3.4e38, -3.4e38,
         1.0000001, -1.0000001, 0.5, 0.5, -0.5, -0.5, 2.0, -2.0],
    ], dtype=torch.float32)
    ones = torch.ones(2, dtype=torch.float32)
    p_edges = ref.quantize_and_pack(edges, ones).numpy()
    const_row = torch.full((1, 16), 0.3, dtype=torch.float32)
    p_const, s_const = ref_pack(ref, const_row)
    np.savez_compressed(os.path.join(HERE, "quant_edges.npz"),
                        w=edges.numpy(), packed=p_edges,
                        w_const=const_row.numpy(), packed_const=p_const,
                        scales_const=s_const)

    E, H, I, Is, T = 4, 64, 128, 128, 5
    g = torch.Generator().manual_seed(4321)
    arrays = {}
    for e in range(E):
        for name, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            w = torch.randn(*shape, generator=g) * 0.02
            p, s = ref_pack(ref, w)
            arrays[f"e{e}_{name}_packed"] = p
            arrays[f"e{e}_{name}_scales"] = s
    for name, shape in (("gate", (Is, H)), ("up", (Is, H)), ("down", (H, Is))):
        w = torch.randn(*shape, generator=g) * 0.02
        p, s = ref_pack(ref, w)
        arrays[f"shared_{name}_packed"] = p
        arrays[f"shared_{name}_scales"] = s
    arrays["gate_w"] = (torch.randn(E, H, generator=g) * 0.02).numpy()
    arrays["x"] = torch.randn(T, H, generator=g).numpy()
    arrays["dims"] = np.array([E, H, I, Is, T], np.int64)
    np.savez_compressed(os.path.join(HERE, "moe_tiny.npz"), **arrays)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../qmoe-rs")
