"""Offline 2-bit packer: the format producer of qmoe-rs (quantize.py:7-33, :97-105).

The packed format every kernel in this package reads is the one qmoe-rs's
quantizer writes:
  * one f32 scale per output row: the unbiased std of the row, clamped to at
    least 1e-5 (quantize.py:98-100);
  * code = clamp(round_half_even(w / scale), -1, 1) + 1, so codes are 0, 1, 2
    (quantize.py:18-22); the runtime also accepts code 3 (value +2,
    src/simd.rs:28-31);
  * four codes per byte, weight j of a group of four in bits 2j..2j+1
    (quantize.py:31), rows of in_features/4 bytes, row-major [out, in/4].

CUDA tensors are packed by the library's device packer (csrc/pack.cu through
qmoe_quantize_pack), bit for bit the same as quantize.py on the host; CPU
tensors by the torch restatement below (the reference's own offline
arithmetic, used to make host-side fixtures).
"""
from __future__ import annotations

import torch

_SHIFTS = (0, 2, 4, 6)


def row_scales(weight: torch.Tensor) -> torch.Tensor:
    """Per-row scale: unbiased std along dim 1, floored at 1e-5."""
    return weight.float().std(dim=1).clamp_min(1e-5)


def ternary_codes(weight: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """int32 codes in {0,1,2} for w / scale rounded half-to-even."""
    q = torch.round(weight.float() / scale.float()[:, None])
    return q.clamp(-1, 1).to(torch.int32) + 1


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """[out, in] int codes (0..3) -> [out, in/4] uint8, LSB-first."""
    out_f, in_f = codes.shape
    if in_f % 4 != 0:
        raise ValueError(f"in_features ({in_f}) must be divisible by 4")
    quads = codes.to(torch.int32).reshape(out_f, in_f // 4, 4)
    packed = torch.zeros((out_f, in_f // 4), dtype=torch.int32, device=codes.device)
    for j, s in enumerate(_SHIFTS):
        packed |= (quads[..., j] & 3) << s
    return packed.to(torch.uint8)


def device_quantize(weight: torch.Tensor, scale: torch.Tensor = None, ctx=None):
    """The device packer (qmoe_quantize_pack) on CUDA tensors, on torch's
    current stream: (packed uint8 [out, in/4], scales f32 [out]); scales
    computed as quantize.py:97-100 unless `scale` is given."""
    from . import capi
    from .layer import default_context
    if not weight.is_cuda:
        raise ValueError("device_quantize takes a CUDA tensor")
    if weight.dim() != 2:
        raise ValueError("weight must be [out_features, in_features]")
    w = weight.float().contiguous()
    out_f, in_f = w.shape
    ctx = ctx or default_context(w.device.index)
    ctx.use_current_torch_stream()
    packed = torch.empty((out_f, in_f // 4), dtype=torch.uint8, device=w.device)
    given = scale is not None
    scales = (scale.to(device=w.device, dtype=torch.float32).contiguous() if given
              else torch.empty(out_f, dtype=torch.float32, device=w.device))
    capi.call("qmoe_quantize_pack", ctx.handle, w.data_ptr(), out_f, in_f, scales.data_ptr(),
              int(given), packed.data_ptr(), capi.QMOE_PTR_DEVICE)
    return packed, scales


def quantize_and_pack(weight: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Same contract as qmoe-rs quantize.py:7-33."""
    if weight.is_cuda:
        return device_quantize(weight, scale)[0]
    return pack_codes(ternary_codes(weight, scale))


def quantize_weight(weight: torch.Tensor):
    """weight [out, in] -> (packed uint8 [out, in/4], scales f32 [out])."""
    if weight.is_cuda:
        return device_quantize(weight)
    scale = row_scales(weight)
    return quantize_and_pack(weight, scale), scale


def unpack_codes(packed: torch.Tensor, in_features: int) -> torch.Tensor:
    """Inverse of pack_codes: [out, in/4] uint8 -> [out, in] int32 codes."""
    p = packed.to(torch.int32)
    cols = [(p >> s) & 3 for s in _SHIFTS]
    return torch.stack(cols, dim=-1).reshape(packed.shape[0], -1)[:, :in_features]
