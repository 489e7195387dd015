"""Parity of the device packer (qmoe_quantize_pack, csrc/pack.cu) with
qmoe-rs's offline quantizer (quantize.py:7-33 and the row scale of :97-100):
packed bytes and f32 scales bit-exact against the committed quantize.py
fixtures and against the same arithmetic on the host (torch CPU), on the
V2-Lite / V3 matrix widths, the unstaged wide-row path, ragged tiny rows,
rounding ties, large means, NaN and inf."""
import ctypes
import os

import numpy as np
import pytest
import torch

from qmoe_b200 import QmoeError, capi, default_context
from qmoe_b200 import quantize as qz

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def host_pack(w: torch.Tensor, scale=None):
    """quantize.py's arithmetic on the host (torch CPU)."""
    if scale is None:
        scale = w.std(dim=1).clamp(min=1e-5)
    return qz.pack_codes(qz.ternary_codes(w, scale)), scale


def same_f32_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bit-equal f32 values; NaN matches NaN whatever its payload (the host's
    inf - inf is x86's negative quiet NaN, the device's the canonical one)."""
    a = a.detach().cpu().contiguous()
    b = b.detach().cpu().contiguous()
    na, nb = torch.isnan(a), torch.isnan(b)
    if not torch.equal(na, nb):
        return False
    return torch.equal(a[~na].view(torch.int32), b[~nb].view(torch.int32))


def test_device_packer_matches_quantize_py_fixtures():
    _cuda()
    z = np.load(os.path.join(GOLDEN, "quant_small.npz"))
    for k in ("a", "b"):
        w = torch.from_numpy(z[f"w_{k}"]).cuda()
        packed, scales = qz.device_quantize(w)
        assert np.array_equal(packed.cpu().numpy(), z[f"packed_{k}"])
        assert np.array_equal(scales.cpu().numpy().view(np.int32), z[f"scales_{k}"].view(np.int32))


def test_device_packer_rounding_edges_and_constant_row():
    _cuda()
    z = np.load(os.path.join(GOLDEN, "quant_edges.npz"))
    w = torch.from_numpy(z["w"]).cuda()
    packed, _ = qz.device_quantize(w, torch.ones(w.shape[0]))
    assert np.array_equal(packed.cpu().numpy(), z["packed"])
    pc, sc = qz.device_quantize(torch.from_numpy(z["w_const"]).cuda())
    assert np.array_equal(pc.cpu().numpy(), z["packed_const"])
    assert np.array_equal(sc.cpu().numpy().view(np.int32), z["scales_const"].view(np.int32))


@pytest.mark.parametrize("out_f,in_f", [
    (1408, 2048),     # V2-Lite gate/up
    (2048, 1408),     # V2-Lite down
    (512, 2816),      # V2-Lite shared down rows
    (96, 7168),       # V3 gate/up rows
    (24, 32768),      # wider than the shared-memory staging limit
    (37, 4), (5, 12), (1, 64),
])
def test_device_packer_bit_exact_vs_host(out_f, in_f):
    _cuda()
    g = torch.Generator().manual_seed(out_f * 131 + in_f)
    w = torch.randn(out_f, in_f, generator=g) * 0.02
    w[: max(1, out_f // 8)] += 3.0                      # rows with a large mean
    p_ref, s_ref = host_pack(w)
    p, s = qz.device_quantize(w.cuda())
    assert same_f32_bits(s, s_ref)
    assert torch.equal(p.cpu(), p_ref)
    # given scales (quantize_and_pack(weight, scale))
    s_in = torch.rand(out_f, generator=g) * 0.05 + 1e-3
    p_ref2, _ = host_pack(w, s_in)
    p2, _ = qz.device_quantize(w.cuda(), s_in)
    assert torch.equal(p2.cpu(), p_ref2)


def test_device_packer_nan_and_inf():
    _cuda()
    w = torch.tensor([[float("nan"), 0.3, -0.7, 2.0, 1.0, 1.0, 1.0, 1.0],
                      [float("inf"), -float("inf"), 0.2, 0.1, 0.5, -0.5, 0.0, 3.0],
                      [0.01, -0.02, 0.03, 0.0, 0.05, -0.06, 0.07, -0.08]])
    ones = torch.ones(3)
    p_ref, _ = host_pack(w, ones)
    p, _ = qz.device_quantize(w.cuda(), ones)
    assert torch.equal(p.cpu(), p_ref)
    p_ref, s_ref = host_pack(w)
    p, s = qz.device_quantize(w.cuda())
    assert same_f32_bits(s, s_ref)
    assert torch.equal(p.cpu(), p_ref)


def test_device_packer_rounding_boundaries():
    """Weights within a few ulps of +-scale/2 (the round-half-even ties of
    w / scale), scales over e^-40..e^40 of both signs, 0, -0, inf and the
    smallest subnormal: the codes of torch's division and rounding."""
    _cuda()
    rng = np.random.default_rng(11)
    R, N = 64, 256
    s = (np.exp(rng.uniform(-40, 40, R)) * rng.choice([-1, 1], R)).astype(np.float32)
    s[:4] = np.array([0.0, -0.0, np.inf, 1e-45], np.float32)
    half = s * np.float32(0.5)
    w = np.empty((R, N), np.float32)
    for j in range(N):
        k = int(rng.integers(-6, 7))
        v = half.copy()
        for _ in range(abs(k)):
            v = np.nextafter(v, np.float32(np.inf) if k > 0 else np.float32(-np.inf))
        w[:, j] = v * np.float32(rng.choice([-1, 1]))
    w[0, 0], w[1, 1], w[2, 2] = np.nan, np.inf, -np.inf
    wt, st = torch.from_numpy(w), torch.from_numpy(s)
    p_ref, _ = host_pack(wt, st)
    p, _ = qz.device_quantize(wt.cuda(), st)
    assert torch.equal(p.cpu(), p_ref)


def test_device_packer_host_buffers():
    _cuda()
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(300, 1408, generator=g) * 0.02).contiguous()
    p_ref, s_ref = host_pack(w)
    packed = np.zeros((300, 352), np.uint8)
    scales = np.zeros(300, np.float32)
    ctx = default_context(0)
    capi.call("qmoe_quantize_pack", ctx.handle, w.data_ptr(), 300, 1408,
              scales.ctypes.data_as(ctypes.c_void_p), 0,
              packed.ctypes.data_as(ctypes.c_void_p), capi.QMOE_PTR_HOST)
    assert np.array_equal(packed, p_ref.numpy())
    assert np.array_equal(scales.view(np.int32), s_ref.numpy().view(np.int32))


def test_device_packer_rejects_bad_shapes():
    _cuda()
    ctx = default_context(0)
    w = torch.zeros(4, 8, device="cuda")
    s = torch.zeros(4, device="cuda")
    p = torch.zeros(4, 2, dtype=torch.uint8, device="cuda")
    for in_f in (6, 0, -4):
        with pytest.raises(QmoeError):
            capi.call("qmoe_quantize_pack", ctx.handle, w.data_ptr(), 4, in_f, s.data_ptr(), 0,
                      p.data_ptr(), capi.QMOE_PTR_DEVICE)
    with pytest.raises(QmoeError):       # misaligned device w
        capi.call("qmoe_quantize_pack", ctx.handle, w.data_ptr() + 4, 1, 4, s.data_ptr(), 0,
                  p.data_ptr(), capi.QMOE_PTR_DEVICE)
    # zero rows: nothing to do
    capi.call("qmoe_quantize_pack", ctx.handle, w.data_ptr(), 0, 8, s.data_ptr(), 0,
              p.data_ptr(), capi.QMOE_PTR_DEVICE)
