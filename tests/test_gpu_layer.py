"""GPU parity of the CUDA path against the CPU oracle, through the C ABI.

Bars (from the project's parity contract):
  * routing indices bit-exact (given the pinned logit order);
  * sigmoid-scored routing weights bit-exact; softmax weights within a few
    ulp (CUDA expf vs glibc expf);
  * layer outputs: max-abs relative error <= 1e-4 for f32 activations,
    <= 2e-2 for bf16 activations (oracle fed the exact bf16 -> f32 upcast).
"""
import os

import numpy as np
import pytest
import torch

import helpers
from helpers import rel_err
from oracle import oracle as qo
from qmoe_b200 import MoEConfig, PackedQMoETensor, QMoELayer, QmoeError, capi
from qmoe_b200 import quantize as qz

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
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


def build(cfg: MoEConfig, seed=1234, bias=None, device="cuda"):
    experts, shared, gate_w = helpers.synth_layer(
        cfg.num_experts, cfg.hidden_dim, cfg.intermediate_dim,
        cfg.shared_intermediate_dim, seed=seed, device=device)
    layer = QMoELayer(cfg, gate_w, experts, shared=shared, bias=bias)
    np_exp = helpers.to_numpy_experts(experts)
    np_sh = helpers.to_numpy_experts([shared])[0] if shared is not None else None
    return layer, np_exp, np_sh, gate_w.cpu().numpy()


def oracle_layer(cfg, gate_w, np_exp, np_sh, x, bias=None):
    return qo.layer_forward(qo_cfg(cfg), gate_w, np_exp, x, shared=np_sh, bias=bias,
                            nthreads=NTHREADS)


# ---------------------------------------------------------------------------
# PackedQMoETensor::forward_simd
# ---------------------------------------------------------------------------

def test_packed_known_answer_on_gpu():
    # src/simd.rs:57-64 on a 64-wide row: byte 0x58 then 0x55 (all code 1 = 0)
    row = np.full(16, 0x55, np.uint8)
    row[0] = 0b01011000
    x = np.zeros((1, 64), np.float32)
    x[0, :4] = [2.0, 3.0, 4.0, 5.0]
    t = PackedQMoETensor.from_bytes(row, (1, 64), np.array([1.5], np.float32))
    y = t.forward_simd(x)
    assert abs(float(y[0, 0]) - 1.5) < 1e-5


@pytest.mark.parametrize("out_f,in_f,batch", [(24, 64, 1), (300, 1408, 3), (2048, 2048, 7),
                                              (129, 192, 33), (1408, 2048, 5)])
def test_packed_forward_matches_oracle(out_f, in_f, batch):
    rng = np.random.default_rng(out_f * 7 + in_f + batch)
    packed = rng.integers(0, 256, (out_f, in_f // 4), dtype=np.uint8)  # code 3 included
    scales = (rng.random(out_f, dtype=np.float32) * 0.05 + 0.01).astype(np.float32)
    x = rng.standard_normal((batch, in_f)).astype(np.float32)
    t = PackedQMoETensor.from_bytes(packed, (out_f, in_f), scales)
    ref = qo.packed_forward(packed, scales, (out_f, in_f), x)
    y_host = t.forward_simd(x)                        # host pointers
    y_dev = t.forward_simd(torch.from_numpy(x).cuda())  # device pointers
    assert rel_err(y_host, ref) <= F32_TOL
    np.testing.assert_array_equal(y_dev.cpu().numpy(), y_host)


def test_packed_forward_ragged_rows_and_large_values():
    rng = np.random.default_rng(5)
    out_f, in_f = 37, 256
    packed = rng.integers(0, 256, (out_f, in_f // 4), dtype=np.uint8)
    scales = rng.random(out_f, dtype=np.float32) + 0.5
    x = (rng.standard_normal((11, in_f)) * 1e4).astype(np.float32)
    x[3] = 0.0                                         # an all-zero row
    x[4, 7] = 3e30                                     # one huge element
    t = PackedQMoETensor.from_bytes(packed, (out_f, in_f), scales)
    y = t.forward_simd(x)
    ref = qo.packed_forward(packed, scales, (out_f, in_f), x)
    for b in range(11):
        assert rel_err(y[b], ref[b]) <= F32_TOL, b
    assert np.all(y[3] == 0.0)


@pytest.mark.parametrize("out_f,in_f,batch", [(40, 100, 3), (130, 1412, 5), (17, 102, 2),
                                              (8, 4, 1), (5, 2, 2), (64, 2047, 33)])
def test_packed_forward_ragged_widths_match_oracle(out_f, in_f, batch):
    # src/tensor.rs:74 reads in_features / 4 bytes per row and src/simd.rs:15
    # ignores the in_features % 4 trailing activations: any width is valid
    rng = np.random.default_rng(out_f + in_f)
    bpr = in_f // 4
    packed = rng.integers(0, 256, (out_f, bpr), dtype=np.uint8)
    scales = (rng.random(out_f, dtype=np.float32) * 0.05 + 0.01).astype(np.float32)
    x = rng.standard_normal((batch, in_f)).astype(np.float32)
    t = PackedQMoETensor.from_bytes(packed.reshape(-1), (out_f, in_f), scales)
    ref = qo.packed_forward(packed, scales, (out_f, in_f), x)
    y_host = t.forward_simd(x)
    y_dev = t.forward_simd(torch.from_numpy(x).cuda()).cpu().numpy()
    if bpr == 0:
        assert np.all(y_host == 0.0) and np.all(ref == 0.0)
    else:
        assert rel_err(y_host, ref) <= F32_TOL
    np.testing.assert_array_equal(y_dev, y_host)
    # a second, larger batch reuses the padded staging rows
    x2 = rng.standard_normal((batch + 9, in_f)).astype(np.float32)
    ref2 = qo.packed_forward(packed, scales, (out_f, in_f), x2)
    y2 = t.forward_simd(x2)
    assert (rel_err(y2, ref2) if bpr else float(np.abs(y2).max())) <= F32_TOL


def test_packed_forward_rejects_bad_shapes():
    with pytest.raises(QmoeError) as ei:
        PackedQMoETensor.from_bytes(np.zeros((4, 25), np.uint8), (0, 100),
                                    np.ones(4, np.float32))
    assert ei.value.code == capi.QMOE_ERR_INVALID
    with pytest.raises(QmoeError) as ei:
        PackedQMoETensor.from_bytes(np.zeros((4, 25), np.uint8), (4, 0),
                                    np.ones(4, np.float32))
    assert ei.value.code == capi.QMOE_ERR_INVALID
    t = PackedQMoETensor.from_bytes(np.zeros((4, 16), np.uint8), (4, 64), np.ones(4, np.float32))
    with pytest.raises(ValueError):
        t.forward_simd(np.zeros((3, 65), np.float32))
    assert t.forward_simd(np.zeros((0, 64), np.float32)).shape == (0, 4)


# ---------------------------------------------------------------------------
# QMoELayer::forward (+ shared expert)
# ---------------------------------------------------------------------------

def test_tiny_fixture_layer_matches_oracle(golden_dir):
    z = np.load(os.path.join(golden_dir, "moe_tiny.npz"))
    E, H, I, Is, T = [int(v) for v in z["dims"]]
    np_exp = [[(z[f"e{e}_{n}_packed"].reshape(-1), z[f"e{e}_{n}_scales"])
               for n in ("gate", "up", "down")] for e in range(E)]
    np_sh = [(z[f"shared_{n}_packed"].reshape(-1), z[f"shared_{n}_scales"])
             for n in ("gate", "up", "down")]
    cfg = MoEConfig(E, 2, H, I, shared_intermediate_dim=Is)
    layer = QMoELayer(cfg, z["gate_w"], np_exp, shared=np_sh)
    out, idx, w = layer.forward(z["x"], return_routing=True)
    ro, ri, rw = oracle_layer(cfg, z["gate_w"], np_exp, np_sh, z["x"])
    np.testing.assert_array_equal(idx, ri)
    np.testing.assert_allclose(w, rw, rtol=1e-6, atol=0)
    assert rel_err(out, ro) <= F32_TOL


@pytest.mark.parametrize("T", [1, 32])
def test_v2_lite_decode_matches_oracle(T):
    cfg = MoEConfig(64, 6, 2048, 1408, shared_intermediate_dim=2816, norm_topk_prob=(T == 32))
    layer, np_exp, np_sh, gw = build(cfg, seed=100 + T)
    x = torch.randn(T, 2048, generator=torch.Generator().manual_seed(T))
    out, idx, w = layer.forward(x.cuda(), return_routing=True)
    ro, ri, rw = oracle_layer(cfg, gw, np_exp, np_sh, x.numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=0)
    assert rel_err(out.cpu().numpy(), ro) <= F32_TOL


def test_host_and_device_pointers_agree_and_are_deterministic():
    cfg = MoEConfig(8, 2, 256, 128, shared_intermediate_dim=192)
    layer, *_ = build(cfg, seed=7)
    x = torch.randn(13, 256, generator=torch.Generator().manual_seed(1))
    a = layer.forward(x)                       # CPU tensor -> host pointers
    b = layer.forward(x.cuda()).cpu()
    c = layer.forward(x.cuda()).cpu()
    np.testing.assert_array_equal(a.numpy(), b.numpy())
    np.testing.assert_array_equal(b.numpy(), c.numpy())


@pytest.mark.parametrize("dtype,T", [(torch.float32, 32), (torch.bfloat16, 7), (torch.float32, 64)])
def test_pinned_host_buffers_read_in_place(dtype, T):
    # page-locked x and out: the front reads x over the bus and leaves the
    # device copy the later kernels use, the combine writes out in place; the
    # result must be the device path's bits, and pageable buffers (staged
    # copies) must agree too
    cfg = MoEConfig(16, 4, 512, 256, shared_intermediate_dim=256)
    layer, *_ = build(cfg, seed=23)
    x = torch.randn(T, 512, generator=torch.Generator().manual_seed(T)).to(dtype)
    ref = layer.forward(x.cuda()).cpu()
    xp = x.pin_memory()
    op = torch.empty_like(xp).pin_memory()
    idx = layer.forward(xp, out=op, return_routing=True)[1]
    assert torch.equal(op, ref)
    _, ridx, _ = layer.forward(x.cuda(), return_routing=True)
    assert torch.equal(idx, ridx.cpu())
    pageable = layer.forward(x.clone())
    assert torch.equal(pageable, ref)


@pytest.mark.parametrize("dtype,T", [(torch.float32, 32), (torch.bfloat16, 5)])
def test_repeated_pinned_forwards_replay_one_graph(dtype, T):
    # the same page-locked x and out over several calls: the second call
    # captures the kernel sequence, later ones replay it; new contents of x
    # must give the device path's new results every time, and a call with
    # another output buffer must not reuse the graph
    cfg = MoEConfig(16, 4, 512, 256, shared_intermediate_dim=256)
    layer, *_ = build(cfg, seed=29)
    xp = torch.empty(T, 512, dtype=dtype).pin_memory()
    op = torch.empty(T, 512, dtype=dtype).pin_memory()
    op2 = torch.empty_like(op).pin_memory()
    # a side stream (the legacy default stream cannot be captured; there the
    # calls run without a graph)
    with torch.cuda.stream(torch.cuda.Stream()):
        for i in range(4):
            x = torch.randn(T, 512, generator=torch.Generator().manual_seed(100 + i)).to(dtype)
            xp.copy_(x)
            ref = layer.forward(x.cuda()).cpu()
            layer.forward(xp, out=op)
            assert torch.equal(op, ref), f"call {i}"
        layer.forward(xp, out=op2)
        assert torch.equal(op2, op)


def test_bf16_activations_within_tolerance():
    cfg = MoEConfig(16, 4, 512, 256, shared_intermediate_dim=256)
    layer, np_exp, np_sh, gw = build(cfg, seed=11)
    x = torch.randn(9, 512, generator=torch.Generator().manual_seed(3)).bfloat16()
    out, idx, _ = layer.forward(x.cuda(), return_routing=True)
    assert out.dtype == torch.bfloat16
    ro, ri, _ = oracle_layer(cfg, gw, np_exp, np_sh, x.float().numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel_err(out.float().cpu().numpy(), ro) <= BF16_TOL


def test_skewed_routing_long_segments():
    # every token picks the same experts: segments of T tokens, many groups
    cfg = MoEConfig(8, 2, 256, 128)
    experts, _, gate_w = helpers.synth_layer(8, 256, 128, seed=5, device="cuda")
    gate_w = gate_w.clone()
    gate_w[3] += 0.5
    gate_w[6] += 0.4
    layer = QMoELayer(cfg, gate_w, experts)
    x = torch.rand(37, 256, generator=torch.Generator().manual_seed(2)) + 0.5
    out, idx, _ = layer.forward(x.cuda(), return_routing=True)
    assert set(np.unique(idx.cpu().numpy())) == {3, 6}
    ro, ri, _ = qo.moe_forward(qo_cfg(cfg), gate_w.cpu().numpy(),
                               helpers.to_numpy_experts(experts), x.numpy(),
                               nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel_err(out.cpu().numpy(), ro) <= F32_TOL


def test_sigmoid_group_limited_routing_bit_exact():
    E, G, TG, k = 32, 8, 4, 8
    cfg = MoEConfig(E, k, 256, 128, scoring=capi.QMOE_SCORING_SIGMOID, n_group=G,
                    topk_group=TG, norm_topk_prob=True, routed_scaling_factor=2.5)
    bias = (torch.randn(E, generator=torch.Generator().manual_seed(8)) * 0.05).float()
    layer, np_exp, _, gw = build(cfg, seed=21, bias=bias.cuda())
    x = torch.randn(19, 256, generator=torch.Generator().manual_seed(4))
    out, idx, w = layer.forward(x.cuda(), return_routing=True)
    ro, ri, rw = qo.moe_forward(qo_cfg(cfg), gw, np_exp, x.numpy(), bias=bias.numpy(),
                                nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(w.cpu().numpy(), rw)
    assert rel_err(out.cpu().numpy(), ro) <= F32_TOL


# Chunk-partials path at three token tilings (T=50: 64-token tiles, ragged;
# T=32 after a large reserve; T=700: many tiles); all must give the same bits.
@pytest.mark.parametrize("T,reserve", [(50, 0), (700, 0), (32, 4096)])
def test_route_only_matches_oracle_bit_exact(T, reserve):
    cfg = MoEConfig(64, 6, 2048, 128)
    experts, _, gw = helpers.synth_layer(64, 2048, 128, seed=3, device="cuda")
    layer = QMoELayer(cfg, gw, experts)
    if reserve:
        layer.reserve(reserve)                 # scratch sized for the big batch
    x = torch.randn(T, 2048, generator=torch.Generator().manual_seed(9))
    idx, w = layer.route(x.cuda())
    logits = qo.gate_logits(x.numpy(), gw.cpu().numpy())
    ri, rw = qo.route(qo_cfg(cfg), logits)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=0)


@pytest.mark.parametrize("E,H,T,dtype,sigmoid", [
    (256, 4096, 2100, torch.float32, True),    # V3-style routing, partials would not fit
    (160, 1024, 3300, torch.bfloat16, False),  # a ragged 128-expert tile, ragged 64-token tile
    (96, 512, 5500, torch.float32, False),     # 96 experts: one tile, 32 of its columns empty
])
def test_large_batch_logits_bit_exact(E, H, T, dtype, sigmoid):
    # T * E >= 2^19 with E > 64: the paired-FP32 tile kernel computes whole
    # logits; they and the routing on them must be the oracle's bits
    if sigmoid:
        cfg = MoEConfig(E, 8, H, 128, scoring=capi.QMOE_SCORING_SIGMOID, n_group=8,
                        topk_group=4, norm_topk_prob=True, routed_scaling_factor=2.5)
    else:
        cfg = MoEConfig(E, 6, H, 128)
    experts, _, gw = helpers.synth_layer(E, H, 128, seed=29 + E, device="cuda")
    layer = QMoELayer(cfg, gw, experts)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(12)).to(dtype)
    idx, w = layer.route(x.cuda())
    logits = qo.gate_logits(x.float().numpy(), gw.cpu().numpy())
    ri, rw = qo.route(qo_cfg(cfg), logits)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    if sigmoid:
        np.testing.assert_array_equal(w.cpu().numpy(), rw)
    else:
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=0)


@pytest.mark.parametrize("T", [19, 1100])
def test_sigmoid_routing_both_logit_paths_bit_exact(T):
    cfg = MoEConfig(32, 8, 256, 128, scoring=capi.QMOE_SCORING_SIGMOID, n_group=8,
                    topk_group=4, norm_topk_prob=True, routed_scaling_factor=2.5)
    experts, _, gw = helpers.synth_layer(32, 256, 128, seed=23, device="cuda")
    layer = QMoELayer(cfg, gw, experts)
    x = torch.randn(T, 256, generator=torch.Generator().manual_seed(T)).bfloat16()
    idx, w = layer.route(x.cuda())
    logits = qo.gate_logits(x.float().numpy(), gw.cpu().numpy())
    ri, rw = qo.route(qo_cfg(cfg), logits)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(w.cpu().numpy(), rw)


@pytest.mark.parametrize("case", ["sigmoid", "sigmoid_minus_inf_bias", "softmax_groups"])
def test_small_batch_selection_with_permute_matches_oracle(case):
    # 32 tokens of 256 experts: the CTA-per-token selection with the permute
    # in its last CTA -- group scores by warp reductions, ranks over the kept
    # groups, or over every expert when fewer than k kept experts score above
    # -inf (the -inf bias case: five finite experts, ties broken by index)
    E, H, I = 256, 512, 128
    bias = None
    if case == "softmax_groups":
        cfg = MoEConfig(E, 6, H, I, n_group=8, topk_group=3)
    else:
        cfg = MoEConfig(E, 8, H, I, scoring=capi.QMOE_SCORING_SIGMOID, n_group=8, topk_group=4,
                        norm_topk_prob=True, routed_scaling_factor=2.5)
        bias = (torch.randn(E, generator=torch.Generator().manual_seed(77)) * 0.05).float()
        if case == "sigmoid_minus_inf_bias":
            bias[:] = float("-inf")
            bias[[3, 40, 41, 200, 201]] = 0.0
    layer, np_exp, _, gw = build(cfg, seed=31, bias=None if bias is None else bias.cuda())
    x = torch.randn(32, H, generator=torch.Generator().manual_seed(5))
    out, idx, w = layer.forward(x.cuda(), return_routing=True)
    ro, ri, rw = qo.moe_forward(qo_cfg(cfg), gw, np_exp, x.numpy(),
                                bias=None if bias is None else bias.numpy(), nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    if case == "softmax_groups":
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=0)
    else:
        np.testing.assert_array_equal(w.cpu().numpy(), rw)
    assert rel_err(out.cpu().numpy(), ro) <= F32_TOL


def test_forward_routed_matches_oracle():
    cfg = MoEConfig(16, 4, 256, 192)
    experts, _, gw = helpers.synth_layer(16, 256, 192, seed=17, device="cuda")
    # an expert-parallel rank owning experts 4..11
    layer = QMoELayer(cfg, gw, experts[4:12], expert_begin=4)
    rng = np.random.default_rng(0)
    R = 23
    idx = np.full((R, 4), -1, np.int32)
    for r in range(R):
        sel = rng.choice(8, size=rng.integers(0, 5), replace=False)
        idx[r, :len(sel)] = sel
    w = rng.random((R, 4), dtype=np.float32)
    x = rng.standard_normal((R, 256)).astype(np.float32)
    out = layer.forward_routed(x, idx, w)
    np_exp = helpers.to_numpy_experts(experts[4:12])
    ref = qo.experts_forward(qo.MoEConfig(8, 4, 256, 192), np_exp, x, idx, w)
    assert rel_err(out, ref) <= F32_TOL
    assert np.all(out[np.all(idx < 0, axis=1)] == 0.0)


def test_shared_forward_and_accumulate():
    cfg = MoEConfig(4, 1, 128, 64, shared_intermediate_dim=320)
    layer, _, np_sh, _ = build(cfg, seed=23)
    x = np.random.default_rng(1).standard_normal((6, 128)).astype(np.float32)
    ref = qo.shared_forward(np_sh, x, 128, 320)
    s = layer.shared_forward(x)
    assert rel_err(s, ref) <= F32_TOL
    base = np.ones((6, 128), np.float32)
    acc = layer.shared_forward(x, out=base.copy())
    assert rel_err(acc - 1.0, ref) <= 1e-4


def test_graph_replay_after_x_copy_reallocated():
    # the cached graph of repeated page-locked forwards reads the layer's
    # device copy of x; a host-pointer call that reallocates that copy must
    # make the next repeat capture again instead of replaying into freed memory
    cfg = MoEConfig(16, 4, 512, 256, shared_intermediate_dim=256)
    layer, *_ = build(cfg, seed=31)
    layer.reserve(1024)
    xp = torch.randn(32, 512, generator=torch.Generator().manual_seed(1)).pin_memory()
    op = torch.empty(32, 512).pin_memory()
    with torch.cuda.stream(torch.cuda.Stream()):
        ref = layer.forward(xp.cuda()).cpu()
        for _ in range(3):                        # second call captures, third replays
            layer.forward(xp, out=op)
            assert torch.equal(op, ref)
        big = torch.randn(64, 512, generator=torch.Generator().manual_seed(2))   # pageable
        layer.forward(big)                        # grows the device copy of x
        xp.copy_(torch.randn(32, 512, generator=torch.Generator().manual_seed(3)))
        ref = layer.forward(xp.cuda()).cpu()
        for _ in range(3):
            layer.forward(xp, out=op)
            assert torch.equal(op, ref)


def test_layer_without_experts_is_its_shared_expert():
    # qmoe-rs: QMoELayer::forward returns zeros for empty `experts`
    # (src/moe.rs:46-48); the block adds the shared expert (src/model.rs:386-389)
    H, Is = 512, 320
    cfg = MoEConfig(8, 2, H, 256, shared_intermediate_dim=Is)
    _, shared, _ = helpers.synth_layer(1, H, 256, Is, seed=8, device="cuda")
    layer = QMoELayer(cfg, None, [], shared=shared)
    np_sh = helpers.to_numpy_experts([shared])[0]
    for dtype, T, tol in ((torch.float32, 5, F32_TOL), (torch.bfloat16, 300, BF16_TOL)):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(dtype)
        out, idx, w = layer.forward(x.cuda(), return_routing=True)
        ref = qo.shared_forward(np_sh, x.float().numpy(), H, Is)
        assert rel_err(out.float().cpu().numpy(), ref) <= tol
        assert torch.all(idx == -1) and torch.all(w == 0)
        host = layer.forward(x)                    # host pointers
        assert torch.equal(host, out.cpu())
    bare = QMoELayer(MoEConfig(8, 2, H, 256), None, [])
    z = bare.forward(torch.randn(7, H, device="cuda"))
    assert torch.all(z == 0)
    zh = bare.forward(np.ones((3, H), np.float32))
    assert np.all(np.asarray(zh) == 0)


def test_empty_batch_is_a_noop():
    cfg = MoEConfig(4, 2, 64, 128)
    layer, *_ = build(cfg, seed=1)
    out = layer.forward(torch.zeros(0, 64, device="cuda"))
    assert out.shape == (0, 64)


def test_invalid_configs_rejected():
    experts, _, gw = helpers.synth_layer(4, 64, 128, seed=1, device="cuda")
    with pytest.raises(QmoeError):
        QMoELayer(MoEConfig(4, 5, 64, 128), gw, experts)          # top_k > E
    with pytest.raises(QmoeError):
        QMoELayer(MoEConfig(4, 2, 64, 128, n_group=3, topk_group=1), gw, experts)
    with pytest.raises(QmoeError):
        QMoELayer(MoEConfig(4, 2, 64, 128, shared_intermediate_dim=64), gw, experts)


def test_quantizer_on_device_matches_host():
    w = torch.randn(64, 256, generator=torch.Generator().manual_seed(0)) * 0.02
    p_cpu, s_cpu = qz.quantize_weight(w)
    p_gpu, s_gpu = qz.quantize_weight(w.cuda())     # the device packer (csrc/pack.cu)
    assert np.array_equal(s_cpu.numpy().view(np.int32), s_gpu.cpu().numpy().view(np.int32))
    assert torch.equal(p_cpu, p_gpu.cpu())


@pytest.mark.parametrize("E,k,H,T,scoring", [
    (64, 6, 2048, 1, capi.QMOE_SCORING_SOFTMAX),      # cluster front, 16 CTAs x 2 chunks
    (64, 6, 2048, 32, capi.QMOE_SCORING_SOFTMAX),     # the decode benchmark's shape
    (64, 6, 2048, 64, capi.QMOE_SCORING_SOFTMAX),     # 4 tokens per CTA of the cluster
    (96, 4, 1024, 20, capi.QMOE_SCORING_SOFTMAX),     # experts not a multiple of 64
    (256, 8, 512, 16, capi.QMOE_SCORING_SIGMOID),     # cluster front, group limit, 8 CTAs
    (256, 8, 512, 17, capi.QMOE_SCORING_SIGMOID),     # too many logits for one cluster:
])                                                    # selection kernel's last CTA permutes
def test_fused_front_matches_separate_router(E, k, H, T, scoring):
    """Small batches route through a fused front (the one-cluster kernel, or
    the selection kernel whose last CTA permutes); route() runs the separate
    router kernels.  Both must give the same bits, and the layer output must
    match the oracle."""
    kw = {}
    if scoring == capi.QMOE_SCORING_SIGMOID:
        kw = dict(scoring=scoring, n_group=8, topk_group=4, norm_topk_prob=True,
                  routed_scaling_factor=2.5)
    cfg = MoEConfig(E, k, H, 128, shared_intermediate_dim=128, **kw)
    layer, np_exp, np_sh, gw = build(cfg, seed=E + T)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(T + 3))
    out, idx, w = layer.forward(x.cuda(), return_routing=True)
    idx2, w2 = layer.route(x.cuda())
    assert torch.equal(idx, idx2) and torch.equal(w, w2)
    ro, ri, rw = oracle_layer(cfg, gw, np_exp, np_sh, x.numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel_err(out.cpu().numpy(), ro) <= F32_TOL


@pytest.mark.parametrize("E,k,H,I,Is,T,dtype", [
    (64, 6, 2048, 1408, 2816, 32, torch.float32),   # the decode benchmark's layer
    (64, 6, 2048, 1408, 2816, 5, torch.bfloat16),
    (16, 4, 512, 256, 0, 300, torch.float32),       # no shared expert; router + permute kernels
    (32, 8, 768, 320, 448, 64, torch.float32),      # rows not multiples of 256
])
def test_cooperative_and_split_decode_agree(E, k, H, I, Is, T, dtype):
    """The decode path makes its activation limbs and the final combine inside
    the two GEMV kernels (cooperative launches); DECODE_SPLIT runs them as
    separate kernels.  Same bits, and the oracle's result within tolerance."""
    cfg = MoEConfig(E, k, H, I, shared_intermediate_dim=Is)
    layer, np_exp, np_sh, gw = build(cfg, seed=E + T)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(dtype)
    xd = x.cuda()
    layer.set_path(capi.QMOE_PATH_DECODE)
    a = layer.forward(xd)
    b = layer.forward(xd)
    layer.set_path(capi.QMOE_PATH_DECODE_SPLIT)
    c = layer.forward(xd)
    layer.set_path(capi.QMOE_PATH_AUTO)
    torch.cuda.synchronize()
    assert torch.equal(a, b), "repeated cooperative forwards differ"
    assert torch.equal(a, c), "cooperative and split decode forwards differ"
    ro, _, _ = oracle_layer(cfg, gw, np_exp, np_sh, x.float().numpy())
    tol = 2e-2 if dtype == torch.bfloat16 else F32_TOL
    assert rel_err(a.float().cpu().numpy(), ro) <= tol
