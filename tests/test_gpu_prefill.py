"""GPU parity of the prefill path (tcgen05 bf16 GEMM over 2-bit weights).

bf16 activations only; the oracle is fed the exact bf16 -> f32 upcast.
Bars: routing indices bit-exact, layer outputs within max-abs relative
error 2e-2.  The prefill kernels round the SwiGLU rows to bf16 and
accumulate in f32 in the tensor core's order, so they are also checked
against the exact integer-limb decode path on the same input.
"""
import os

import numpy as np
import pytest
import torch

import helpers
from helpers import rel_err
from oracle import oracle as qo
from qmoe_b200 import MoEConfig, QMoELayer, QmoeError, capi

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
NTHREADS = max(1, min(8, os.cpu_count() or 1))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def qo_cfg(cfg: MoEConfig) -> qo.MoEConfig:
    return qo.MoEConfig(cfg.num_experts, cfg.top_k, cfg.hidden_dim, cfg.intermediate_dim,
                        cfg.shared_intermediate_dim, cfg.scoring, cfg.n_group,
                        cfg.topk_group, cfg.norm_topk_prob, cfg.routed_scaling_factor)


def build(cfg: MoEConfig, seed=1234, gate_shift=None):
    experts, shared, gate_w = helpers.synth_layer(
        cfg.num_experts, cfg.hidden_dim, cfg.intermediate_dim,
        cfg.shared_intermediate_dim, seed=seed, device="cuda")
    if gate_shift is not None:
        gate_w = gate_w + gate_shift.to(gate_w.device)[:, None]
    layer = QMoELayer(cfg, gate_w, experts, shared=shared)
    np_exp = helpers.to_numpy_experts(experts)
    np_sh = helpers.to_numpy_experts([shared])[0] if shared is not None else None
    return layer, np_exp, np_sh, gate_w.cpu().numpy()


def bf16_input(T, H, seed):
    return torch.randn(T, H, generator=torch.Generator().manual_seed(seed)).bfloat16()


def run_both_paths(layer, x):
    layer.set_path(capi.QMOE_PATH_PREFILL)
    out_p, idx_p, _ = layer.forward(x.cuda(), return_routing=True)
    layer.set_path(capi.QMOE_PATH_DECODE)
    out_d, idx_d, _ = layer.forward(x.cuda(), return_routing=True)
    layer.set_path(capi.QMOE_PATH_AUTO)
    return out_p.float().cpu().numpy(), idx_p.cpu().numpy(), out_d.float().cpu().numpy(), \
        idx_d.cpu().numpy()


@pytest.mark.parametrize("E,k,H,I,Is,T", [
    (8, 2, 256, 128, 192, 100),      # ragged groups (counts not multiples of 16)
    (4, 2, 128, 64, 0, 7),           # tiny, no shared expert, one 16-column tile
    (16, 4, 512, 320, 256, 333),     # I not a multiple of 256 (ragged weight stage)
])
def test_prefill_matches_oracle(E, k, H, I, Is, T):
    cfg = MoEConfig(E, k, H, I, shared_intermediate_dim=Is)
    layer, np_exp, np_sh, gw = build(cfg, seed=E * 100 + T)
    x = bf16_input(T, H, T)
    out_p, idx_p, out_d, idx_d = run_both_paths(layer, x)
    ro, ri, _ = qo.layer_forward(qo_cfg(cfg), gw, np_exp, x.float().numpy(), shared=np_sh,
                                 nthreads=NTHREADS)
    np.testing.assert_array_equal(idx_p, ri)
    np.testing.assert_array_equal(idx_d, ri)
    assert rel_err(out_p, ro) <= BF16_TOL
    assert rel_err(out_d, ro) <= BF16_TOL
    assert rel_err(out_p, out_d) <= BF16_TOL


def test_prefill_long_segments_split_into_groups():
    # two experts take every token: segments of 600 positions = 3 groups each
    cfg = MoEConfig(8, 2, 256, 128, shared_intermediate_dim=128)
    shift = torch.zeros(8)
    shift[2], shift[5] = 0.5, 0.4
    layer, np_exp, np_sh, gw = build(cfg, seed=9, gate_shift=shift)
    x = (torch.rand(600, 256, generator=torch.Generator().manual_seed(3)) + 0.5).bfloat16()
    out_p, idx_p, out_d, _ = run_both_paths(layer, x)
    assert set(np.unique(idx_p)) == {2, 5}
    ro, ri, _ = qo.layer_forward(qo_cfg(cfg), gw, np_exp, x.float().numpy(), shared=np_sh,
                                 nthreads=NTHREADS)
    np.testing.assert_array_equal(idx_p, ri)
    assert rel_err(out_p, ro) <= BF16_TOL
    assert rel_err(out_p, out_d) <= BF16_TOL


def test_prefill_v2_lite_shape_matches_oracle():
    # configs[2] layer shape (hidden 2048, 64 experts, top-6, expert 1408,
    # shared 2816) at a batch the oracle finishes in seconds
    cfg = MoEConfig(64, 6, 2048, 1408, shared_intermediate_dim=2816)
    layer, np_exp, np_sh, gw = build(cfg, seed=77)
    x = bf16_input(96, 2048, 5)
    layer.set_path(capi.QMOE_PATH_PREFILL)
    out, idx, _ = layer.forward(x.cuda(), return_routing=True)
    ro, ri, _ = qo.layer_forward(qo_cfg(cfg), gw, np_exp, x.float().numpy(), shared=np_sh,
                                 nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel_err(out.float().cpu().numpy(), ro) <= BF16_TOL


def test_prefill_full_configs2_agrees_with_exact_path():
    # configs[2] at full size (2048 bf16 tokens): the prefill GEMM against
    # the exact integer-limb path on the same input (size-independent check),
    # and against the oracle on a seeded sample of the batch's tokens (each
    # token's output row depends on that token alone)
    cfg = MoEConfig(64, 6, 2048, 1408, shared_intermediate_dim=2816)
    layer, np_exp, np_sh, gw = build(cfg, seed=4242)
    x = torch.randn(2048, 2048, generator=torch.Generator().manual_seed(11)).bfloat16()
    out_p, idx_p, out_d, idx_d = run_both_paths(layer, x)
    np.testing.assert_array_equal(idx_p, idx_d)
    assert rel_err(out_p, out_d) <= BF16_TOL
    assert np.isfinite(out_p).all()
    sample = np.sort(np.random.default_rng(12).choice(2048, 48, replace=False))
    ro, ri, _ = qo.layer_forward(qo_cfg(cfg), gw, np_exp, x[sample].float().numpy(), shared=np_sh,
                                 nthreads=NTHREADS)
    np.testing.assert_array_equal(idx_p[sample], ri)
    assert rel_err(out_p[sample], ro) <= BF16_TOL


def test_prefill_auto_selects_and_is_deterministic():
    cfg = MoEConfig(8, 2, 256, 128, shared_intermediate_dim=192)
    layer, *_ = build(cfg, seed=31)
    x = bf16_input(256, 256, 2).cuda()     # 64 positions per expert -> prefill
    a = layer.forward(x).float().cpu().numpy()
    layer.set_path(capi.QMOE_PATH_PREFILL)
    b = layer.forward(x).float().cpu().numpy()
    c = layer.forward(x).float().cpu().numpy()
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(b, c)


def test_prefill_shared_only_and_routed_entry_points():
    cfg = MoEConfig(16, 4, 256, 192, shared_intermediate_dim=320)
    experts, shared, gw = helpers.synth_layer(16, 256, 192, 320, seed=17, device="cuda")
    layer = QMoELayer(cfg, gw, experts[4:12], expert_begin=4, shared=shared)
    layer.set_path(capi.QMOE_PATH_PREFILL)
    rng = np.random.default_rng(0)
    R = 150
    idx = np.full((R, 4), -1, np.int32)
    for r in range(R):
        sel = rng.choice(8, size=rng.integers(0, 5), replace=False)
        idx[r, :len(sel)] = sel
    w = rng.random((R, 4), dtype=np.float32)
    x = torch.from_numpy(rng.standard_normal((R, 256)).astype(np.float32)).bfloat16()
    out = layer.forward_routed(x.cuda(), torch.from_numpy(idx).cuda(),
                               torch.from_numpy(w).cuda()).float().cpu().numpy()
    np_exp = helpers.to_numpy_experts(experts[4:12])
    ref = qo.experts_forward(qo.MoEConfig(8, 4, 256, 192), np_exp, x.float().numpy(), idx, w)
    assert rel_err(out, ref) <= BF16_TOL
    assert np.all(out[np.all(idx < 0, axis=1)] == 0.0)
    np_sh = helpers.to_numpy_experts([shared])[0]
    s = layer.shared_forward(x.cuda()).float().cpu().numpy()
    sref = qo.shared_forward(np_sh, x.float().numpy(), 256, 320)
    assert rel_err(s, sref) <= BF16_TOL


def test_prefill_rejects_f32_and_bad_shapes():
    cfg = MoEConfig(4, 2, 128, 64)
    layer, *_ = build(cfg, seed=3)
    layer.set_path(capi.QMOE_PATH_PREFILL)
    with pytest.raises(QmoeError):
        layer.forward(torch.randn(40, 128, device="cuda"))        # f32 activations
    cfg2 = MoEConfig(4, 2, 64, 128)                               # hidden % 128 != 0
    layer2, *_ = build(cfg2, seed=3)
    with pytest.raises(QmoeError):
        layer2.set_path(capi.QMOE_PATH_PREFILL)
    with pytest.raises(QmoeError):
        layer2.set_path(7)
