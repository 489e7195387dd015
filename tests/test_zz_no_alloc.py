"""GPU test of qmoe_packed_forward_noalloc, the allocation-free GEMV entry point.

That entry point serves callers that may not allocate device memory, such as
a host program that keeps all HBM in its own pool and passes a plugin only
the buffers of each call.  It must give the same product as the regular
qmoe_packed_forward, call after call, with its work list living in a fixed
device array shared by all calls.

This file is named so that pytest collects it last; it also runs on its own
in a fresh process, where its first call performs the per-device set-up.
"""
import ctypes

import numpy as np
import pytest
import torch

from qmoe_b200 import PackedQMoETensor, QmoeError, capi

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4  # max-abs relative error bar of the f32 parity tests


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _noalloc(packed, scales, shape, x, y):
    out_f, in_f = shape
    capi.call("qmoe_packed_forward_noalloc", 0,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
              _ptr(packed), _ptr(scales), out_f, in_f, _ptr(x), x.shape[0], _ptr(y))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def test_noalloc_matches_packed_forward_on_two_calls():
    rng = np.random.default_rng(2024)
    cases = [((1408, 2048), 37), ((300, 1408), 5)]  # second call: other shape, smaller list
    for (out_f, in_f), batch in cases:
        packed_np = rng.integers(0, 256, (out_f, in_f // 4), dtype=np.uint8)
        scales_np = (rng.random(out_f, dtype=np.float32) * 0.05 + 0.01).astype(np.float32)
        x = torch.from_numpy(rng.standard_normal((batch, in_f)).astype(np.float32)).cuda()
        ref = PackedQMoETensor.from_bytes(packed_np, (out_f, in_f), scales_np).forward_simd(x)
        packed = torch.from_numpy(packed_np).cuda()
        scales = torch.from_numpy(scales_np).cuda()
        for call in range(2):
            y = torch.full((batch, out_f), float("nan"), device="cuda")
            _noalloc(packed, scales, (out_f, in_f), x, y)
            torch.cuda.synchronize()
            assert torch.isfinite(y).all(), (out_f, in_f, call)
            assert _rel_err(y, ref) <= F32_TOL, (out_f, in_f, call)


def test_noalloc_rejects_sizes_beyond_its_limits():
    packed = torch.zeros((8, 16), dtype=torch.uint8, device="cuda")
    scales = torch.ones(8, device="cuda")
    big = torch.zeros((capi.QMOE_NOALLOC_MAX_BATCH + 1, 64), device="cuda")
    y = torch.empty((big.shape[0], 8), device="cuda")
    with pytest.raises(QmoeError) as ei:
        _noalloc(packed, scales, (8, 64), big, y)
    assert ei.value.code == capi.QMOE_ERR_INVALID
    assert "QMOE_NOALLOC_MAX_BATCH" in str(ei.value)
    wide = torch.zeros((2, capi.QMOE_NOALLOC_MAX_IN_FEATURES + 64), device="cuda")
    with pytest.raises(QmoeError) as ei:
        _noalloc(torch.zeros((8, wide.shape[1] // 4), dtype=torch.uint8, device="cuda"),
                 scales, (8, wide.shape[1]), wide, torch.empty((2, 8), device="cuda"))
    assert ei.value.code == capi.QMOE_ERR_INVALID
