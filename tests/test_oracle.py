"""CPU tests of the oracle: pinned against qmoe-rs's own known answers and
fixtures, and cross-checked against the independent Python restatement."""
import os

import numpy as np
import pytest
import torch

import pyref
from oracle import oracle as qo
from qmoe_b200 import quantize as qz


def load_tiny(golden_dir):
    z = np.load(os.path.join(golden_dir, "moe_tiny.npz"))
    E, H, I, Is, T = [int(v) for v in z["dims"]]
    experts = [tuple((z[f"e{e}_{n}_packed"].reshape(-1), z[f"e{e}_{n}_scales"])
                     for n in ("gate", "up", "down")) for e in range(E)]
    shared = tuple((z[f"shared_{n}_packed"].reshape(-1), z[f"shared_{n}_scales"])
                   for n in ("gate", "up", "down"))
    return dict(E=E, H=H, I=I, Is=Is, T=T, experts=experts, shared=shared,
                gate_w=z["gate_w"], x=z["x"])


# --- known answers from qmoe-rs ------------------------------------------

def test_simd_known_answer():
    # src/simd.rs:57-64: byte 0b01011000 -> weights [-1, 1, 0, 0],
    # activations [2, 3, 4, 5], scale 1.5 -> 1.5 (within 1e-5)
    r = qo.dequant_dot(np.array([0b01011000], np.uint8),
                       np.array([2.0, 3.0, 4.0, 5.0], np.float32), 1.5)
    assert abs(r - 1.5) < 1e-5
    assert r == 1.5


def test_code_three_is_plus_two():
    # src/simd.rs:22-31 maps code 0b11 to 3 - 1 = +2.0 (the bench bytes of
    # benches/moe_layer.rs:18-21 contain it, e.g. 0b10100111's low bits)
    r = qo.dequant_dot(np.array([0b11111111], np.uint8),
                       np.array([1.0, 2.0, 3.0, 4.0], np.float32), 1.0)
    assert r == 20.0


def test_ragged_activation_tail_ignored():
    # src/simd.rs:15: num_bytes = min(bytes, act.len() / 4)
    r = qo.dequant_dot(np.array([0xAA, 0xAA], np.uint8),
                       np.array([1, 1, 1, 1, 5, 5], np.float32), 1.0)
    assert r == 4.0


def test_quantizer_matches_reference_fixtures(golden_dir):
    z = np.load(os.path.join(golden_dir, "quant_small.npz"))
    for s in ("a", "b"):
        w = torch.from_numpy(z[f"w_{s}"])
        packed, scales = qz.quantize_weight(w)
        np.testing.assert_array_equal(scales.numpy(), z[f"scales_{s}"])
        np.testing.assert_array_equal(packed.numpy(), z[f"packed_{s}"])
        codes = qz.unpack_codes(packed, w.shape[1])
        assert int(codes.max()) <= 2 and int(codes.min()) >= 0


def test_quantizer_rounding_edges(golden_dir):
    z = np.load(os.path.join(golden_dir, "quant_edges.npz"))
    w = torch.from_numpy(z["w"])
    packed = qz.quantize_and_pack(w, torch.ones(w.shape[0]))
    np.testing.assert_array_equal(packed.numpy(), z["packed"])
    pc, sc = qz.quantize_weight(torch.from_numpy(z["w_const"]))
    np.testing.assert_array_equal(sc.numpy(), z["scales_const"])
    np.testing.assert_array_equal(pc.numpy(), z["packed_const"])
    assert float(sc[0]) == np.float32(1e-5)


# --- oracle vs the independent Python restatement -------------------------

@pytest.mark.parametrize("pairwise", [False, True])
def test_dequant_dot_matches_pyref(pairwise):
    rng = np.random.default_rng(7)
    packed = rng.integers(0, 256, 48, dtype=np.uint8)   # includes code 3
    act = rng.standard_normal(192).astype(np.float32)
    mode = qo.REDUCE_PAIRWISE if pairwise else qo.REDUCE_ORDERED
    a = qo.dequant_dot(packed, act, 0.37, mode)
    b = pyref.dequant_dot(packed, act, np.float32(0.37), pairwise)
    assert np.float32(a) == b


def test_packed_forward_matches_pyref():
    rng = np.random.default_rng(3)
    out_f, in_f, B = 12, 32, 3
    packed = rng.integers(0, 256, out_f * in_f // 4, dtype=np.uint8)
    scales = rng.random(out_f, dtype=np.float32) + 0.5
    x = rng.standard_normal((B, in_f)).astype(np.float32)
    np.testing.assert_array_equal(qo.packed_forward(packed, scales, (out_f, in_f), x),
                                  pyref.packed_forward(packed, scales, (out_f, in_f), x))


def test_reference_bench_generators():
    # deterministic data of benches/moe_layer.rs:11-36, :68-73
    out_f, in_f = 16, 64
    cyc = np.array([0b01011000, 0b10100111, 0b00101110, 0b11100100], np.uint8)
    packed = np.resize(cyc, out_f * in_f // 4)
    scales = (np.sin(np.arange(out_f, dtype=np.float32) * np.float32(0.05))
              + np.float32(1.0)).astype(np.float32)
    x = (np.sin(np.arange(2 * in_f, dtype=np.float32) * np.float32(0.1))
         + np.float32(0.5)).astype(np.float32).reshape(2, in_f)
    np.testing.assert_array_equal(qo.packed_forward(packed, scales, (out_f, in_f), x),
                                  pyref.packed_forward(packed, scales, (out_f, in_f), x))


def test_gate_logits_pinned_order():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 192)).astype(np.float32)
    gw = (rng.standard_normal((5, 192)) * 0.02).astype(np.float32)
    np.testing.assert_array_equal(qo.gate_logits(x, gw), pyref.gate_logits(x, gw))


def test_softmax_routing_matches_pyref():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((6, 16)).astype(np.float32)
    logits[0, 3] = logits[0, 9] = logits[0, 12] = 4.0     # ties -> lower index
    logits[1, :] = 0.0                                   # all tied
    cfg = qo.MoEConfig(16, 4, 64, 128)
    idx, w = qo.route(cfg, logits)
    ridx, rw = pyref.route_softmax(logits, 4)
    np.testing.assert_array_equal(idx, ridx)
    np.testing.assert_array_equal(w, rw)
    assert list(idx[0, :3]) == [3, 9, 12]
    assert list(idx[1]) == [0, 1, 2, 3]


def test_moe_forward_matches_pyref(golden_dir):
    d = load_tiny(golden_dir)
    cfg = qo.MoEConfig(d["E"], 2, d["H"], d["I"])
    out, idx, w = qo.moe_forward(cfg, d["gate_w"], d["experts"], d["x"])
    ro, ri, rw = pyref.moe_forward(d["E"], 2, d["H"], d["I"], d["gate_w"],
                                   d["experts"], d["x"])
    np.testing.assert_array_equal(idx, ri)
    np.testing.assert_array_equal(w, rw)
    np.testing.assert_array_equal(out, ro)


def test_threaded_oracle_is_bit_identical(golden_dir):
    d = load_tiny(golden_dir)
    cfg = qo.MoEConfig(d["E"], 3, d["H"], d["I"], shared_intermediate_dim=d["Is"])
    rng = np.random.default_rng(9)
    x = rng.standard_normal((17, d["H"])).astype(np.float32)
    a = qo.layer_forward(cfg, d["gate_w"], d["experts"], x, shared=d["shared"],
                         nthreads=1)
    b = qo.layer_forward(cfg, d["gate_w"], d["experts"], x, shared=d["shared"],
                         nthreads=4)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)


def test_layer_adds_shared_after_routed(golden_dir):
    # src/model.rs:386-389: moe_out + shared_out, elementwise f32
    d = load_tiny(golden_dir)
    cfg = qo.MoEConfig(d["E"], 2, d["H"], d["I"], shared_intermediate_dim=d["Is"])
    routed, _, _ = qo.moe_forward(cfg, d["gate_w"], d["experts"], d["x"])
    shared = qo.shared_forward(d["shared"], d["x"], d["H"], d["Is"])
    full, _, _ = qo.layer_forward(cfg, d["gate_w"], d["experts"], d["x"],
                                  shared=d["shared"])
    np.testing.assert_array_equal(full, routed + shared)


def test_empty_and_single_token(golden_dir):
    d = load_tiny(golden_dir)
    cfg = qo.MoEConfig(d["E"], 2, d["H"], d["I"])
    out, idx, _ = qo.moe_forward(cfg, d["gate_w"], d["experts"], d["x"][:0])
    assert out.shape == (0, d["H"]) and idx.shape == (0, 2)
    out1, _, _ = qo.moe_forward(cfg, d["gate_w"], d["experts"], d["x"][:1])
    full, _, _ = qo.moe_forward(cfg, d["gate_w"], d["experts"], d["x"])
    np.testing.assert_array_equal(out1[0], full[0])


# --- extension spec (not in qmoe-rs) --------------------------------------

def test_qexp_accuracy():
    xs = np.concatenate([np.linspace(-103, 88.7, 20001, dtype=np.float32),
                         np.float32([0.0, -0.0, 1e-30, -1e-30, 0.5, -0.5])])
    got = np.array([qo.qexp(float(v)) for v in xs], np.float64)
    want = np.exp(xs.astype(np.float64))
    normal = want > np.finfo(np.float32).tiny
    ulp = np.spacing(want[normal].astype(np.float32)).astype(np.float64)
    err = np.abs(got[normal] - want[normal]) / ulp
    assert err.max() <= 2.0, err.max()
    assert qo.qexp(100.0) == np.inf and qo.qexp(-200.0) == 0.0


def _pyroute_sigmoid(logits, bias, k, G, TG, norm, rsf):
    E = logits.shape[0]
    s = np.array([qo.sigmoid(float(v)) for v in logits], np.float32)
    ch = (s + bias).astype(np.float32) if bias is not None else s.copy()
    per = E // G
    gs = []
    for g in range(G):
        c = sorted([(float(ch[g * per + j]), g * per + j) for j in range(per)],
                   key=lambda p: (-p[0], p[1]))
        gs.append(np.float32(np.float32(c[0][0]) + np.float32(c[1][0])))
    gorder = sorted(range(G), key=lambda g: (-gs[g], g))[:TG]
    cand = [e for g in gorder for e in range(g * per, (g + 1) * per)]
    sel = sorted(cand, key=lambda e: (-ch[e], e))[:k]
    w = np.array([s[e] for e in sel], np.float32)
    if norm:
        den = np.float32(0.0)
        for v in w:
            den = np.float32(den + v)
        den = np.float32(den + np.float32(1e-20))
        w = (w / den).astype(np.float32)
    if rsf != 1.0:
        w = (w * np.float32(rsf)).astype(np.float32)
    return np.array(sel, np.int32), w


def test_sigmoid_group_routing_spec():
    rng = np.random.default_rng(21)
    E, G, TG, k = 32, 8, 4, 8
    logits = rng.standard_normal((7, E)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    logits[2, :] = 0.0
    cfg = qo.MoEConfig(E, k, 64, 128, scoring=qo.SCORING_SIGMOID, n_group=G,
                       topk_group=TG, norm_topk_prob=True,
                       routed_scaling_factor=2.5)
    idx, w = qo.route(cfg, logits, bias)
    for t in range(logits.shape[0]):
        ri, rw = _pyroute_sigmoid(logits[t], bias, k, G, TG, True, 2.5)
        np.testing.assert_array_equal(idx[t], ri)
        np.testing.assert_array_equal(w[t], rw)


def test_softmax_renorm_flag():
    rng = np.random.default_rng(2)
    logits = rng.standard_normal((4, 64)).astype(np.float32)
    base = qo.MoEConfig(64, 6, 64, 128)
    i0, w0 = qo.route(base, logits)
    i1, w1 = qo.route(qo.MoEConfig(64, 6, 64, 128, norm_topk_prob=True), logits)
    np.testing.assert_array_equal(i0, i1)
    for t in range(4):
        den = np.float32(0.0)
        for v in w0[t]:
            den = np.float32(den + v)
        den = np.float32(den + np.float32(1e-20))
        np.testing.assert_array_equal(w1[t], (w0[t] / den).astype(np.float32))


def test_invalid_routing_rejected():
    with pytest.raises(ValueError):
        qo.route(qo.MoEConfig(4, 5, 64, 128), np.zeros((1, 4), np.float32))


def test_oracle_layernorm_against_float64_reference():
    # the pinned-order LayerNorm of the oracle (post_attention_layernorm,
    # src/model.rs:366-367) is a LayerNorm: within f32 rounding of torch's
    # float64 result; its bf16 rounding is round-to-nearest-even
    import torch
    rng = np.random.default_rng(3)
    for H in (64, 512, 7168):
        x = (rng.standard_normal((7, H)) * 3 + 1.5).astype(np.float32)
        w = rng.standard_normal(H).astype(np.float32)
        b = rng.standard_normal(H).astype(np.float32)
        y = qo.layernorm(x, w, b, 1e-6)
        ref = torch.nn.functional.layer_norm(torch.from_numpy(x).double(), (H,), torch.from_numpy(w).double(),
                                             torch.from_numpy(b).double(), eps=1e-6).numpy()
        assert np.max(np.abs(y - ref)) <= 2e-5 * max(1.0, np.max(np.abs(ref)))
        yb = qo.layernorm(x, w, b, 1e-6, round_bf16=True)
        assert np.array_equal(yb, torch.from_numpy(y).bfloat16().float().numpy())
