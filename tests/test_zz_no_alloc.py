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

from oracle import oracle as qo
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
        x_np = rng.standard_normal((batch, in_f)).astype(np.float32)
        x = torch.from_numpy(x_np).cuda()
        ref = PackedQMoETensor.from_bytes(packed_np, (out_f, in_f), scales_np).forward_simd(x)
        oracle = torch.from_numpy(qo.packed_forward(packed_np, scales_np, (out_f, in_f), x_np))
        packed = torch.from_numpy(packed_np).cuda()
        scales = torch.from_numpy(scales_np).cuda()
        for call in range(2):
            y = torch.full((batch, out_f), float("nan"), device="cuda")
            _noalloc(packed, scales, (out_f, in_f), x, y)
            torch.cuda.synchronize()
            assert torch.isfinite(y).all(), (out_f, in_f, call)
            assert _rel_err(y, ref) <= F32_TOL, (out_f, in_f, call)
            assert _rel_err(y, oracle) <= F32_TOL, (out_f, in_f, call)


def test_noalloc_allocates_nothing_and_keeps_the_current_device():
    rng = np.random.default_rng(7)
    shapes = [((512, 1024), 3), ((2048, 8192), 40), ((64, 64), 1), ((1408, 2048), 600)]
    bufs = []
    for (out_f, in_f), batch in shapes:
        packed = torch.from_numpy(rng.integers(0, 256, (out_f, in_f // 4), dtype=np.uint8)).cuda()
        scales = torch.from_numpy(rng.random(out_f, dtype=np.float32) + 0.5).cuda()
        x = torch.from_numpy(rng.standard_normal((batch, in_f)).astype(np.float32)).cuda()
        bufs.append((packed, scales, (out_f, in_f), x, torch.empty((batch, out_f), device="cuda")))
    _noalloc(*bufs[0])                      # set-up done (or done earlier)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    dev0 = torch.cuda.current_device()
    for _ in range(3):
        for b in bufs:
            _noalloc(*b)
            assert torch.cuda.current_device() == dev0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device memory changed by {free0 - free1} bytes"


def test_noalloc_leaves_wider_regular_tensors_working():
    # a regular packed tensor wider than the no-allocation limit needs a
    # larger shared-memory opt-in of the same kernel; a no-allocation call in
    # between must not lower it
    rng = np.random.default_rng(11)
    out_f, in_f = 96, 10944
    packed_np = rng.integers(0, 256, (out_f, in_f // 4), dtype=np.uint8)
    scales_np = (rng.random(out_f, dtype=np.float32) + 0.5).astype(np.float32)
    x_np = rng.standard_normal((3, in_f)).astype(np.float32)
    t = PackedQMoETensor.from_bytes(packed_np, (out_f, in_f), scales_np)
    ref = torch.from_numpy(qo.packed_forward(packed_np, scales_np, (out_f, in_f), x_np))
    assert _rel_err(torch.from_numpy(np.asarray(t.forward_simd(x_np))), ref) <= F32_TOL
    small = torch.zeros((8, 16), dtype=torch.uint8, device="cuda")
    y = torch.empty((2, 8), device="cuda")
    _noalloc(small, torch.ones(8, device="cuda"), (8, 64), torch.zeros((2, 64), device="cuda"), y)
    torch.cuda.synchronize()
    assert _rel_err(torch.from_numpy(np.asarray(t.forward_simd(x_np))), ref) <= F32_TOL


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
