"""GPU parity at the DeepSeek-V3 layer shape of the benchmark:
hidden 7168, 256 routed experts, sigmoid scoring with 8 groups of which 4 are
kept, top-8 with renormalised weights scaled by 2.5, one shared expert of
width 2048, experts of width 2048.

The whole 4096-token bf16 batch runs on the GPU; routing is per token, so the
oracle checks a seeded sample of the batch's tokens (their rows of the
output depend on nothing else).  Bars: routing indices and sigmoid weights
bit-exact, outputs within max-abs relative error 2e-2 (bf16) and 1e-4 (f32).
"""
import os

import numpy as np
import pytest
import torch

import helpers
from helpers import rel_err
from oracle import oracle as qo
from qmoe_b200 import MoEConfig, QMoELayer, capi

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2
NTHREADS = max(1, min(16, os.cpu_count() or 1))

E, K, H, I, IS = 256, 8, 7168, 2048, 2048


@pytest.fixture(scope="module")
def v3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=IS, scoring=capi.QMOE_SCORING_SIGMOID,
                    n_group=8, topk_group=4, norm_topk_prob=True, routed_scaling_factor=2.5)
    experts, shared, gate_w = helpers.synth_layer(E, H, I, IS, seed=3333, device="cuda")
    layer = QMoELayer(cfg, gate_w, experts, shared=shared)
    np_exp = helpers.to_numpy_experts(experts)
    np_sh = helpers.to_numpy_experts([shared])[0]
    del experts, shared
    ocfg = qo.MoEConfig(E, K, H, I, IS, scoring=qo.SCORING_SIGMOID, n_group=8, topk_group=4,
                        norm_topk_prob=True, routed_scaling_factor=2.5)
    yield layer, np_exp, np_sh, gate_w.cpu().numpy(), ocfg
    layer.close()
    torch.cuda.empty_cache()


def test_v3_prefill_batch_sampled_tokens_match_oracle(v3):
    layer, np_exp, np_sh, gw, ocfg = v3
    T = 4096
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(41)).bfloat16()
    out, idx, w = layer.forward(x.cuda(), return_routing=True)      # auto: prefill GEMMs
    torch.cuda.synchronize()
    sample = np.sort(np.random.default_rng(7).choice(T, 40, replace=False))
    xs = x[sample].float().numpy()
    ro, ri, rw = qo.layer_forward(ocfg, gw, np_exp, xs, shared=np_sh, nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy()[sample], ri)
    np.testing.assert_array_equal(w.cpu().numpy()[sample], rw)
    assert rel_err(out.float().cpu().numpy()[sample], ro) <= BF16_TOL
    # the same forward twice gives the same bits
    out2 = layer.forward(x.cuda())
    assert torch.equal(out, out2)


def test_v3_prefill_repeated_forwards_bit_identical(v3):
    # The expert path is free of timing-dependent reads: the same 4096-token
    # forward, repeated, gives the same bits every time.  (A pipeline race
    # in an earlier stage geometry of the prefill GEMM changed one expert's
    # rows by 1-2 bf16 ulps in about one forward of 150; 300 forwards catch
    # that rate with probability ~0.86.)
    layer, *_ = v3
    x = torch.randn(4096, H, generator=torch.Generator().manual_seed(45)).bfloat16().cuda()
    idx, w = layer.route(x)
    ref = layer.forward_routed(x, idx, w).clone()
    full = layer.forward(x).clone()
    for i in range(300):
        assert torch.equal(layer.forward_routed(x, idx, w), ref), f"forward_routed {i} differs"
    for i in range(50):
        assert torch.equal(layer.forward(x), full), f"forward {i} differs"


def test_v3_prefill_batch_agrees_with_exact_path_everywhere(v3):
    # every token of a 1024-token batch: prefill GEMMs against the exact
    # integer-limb GEMV path (a size-independent cross-check of the rest)
    layer, *_ = v3
    x = torch.randn(1024, H, generator=torch.Generator().manual_seed(43)).bfloat16().cuda()
    layer.set_path(capi.QMOE_PATH_PREFILL)
    a, ia, _ = layer.forward(x, return_routing=True)
    layer.set_path(capi.QMOE_PATH_DECODE)
    b, ib, _ = layer.forward(x, return_routing=True)
    layer.set_path(capi.QMOE_PATH_AUTO)
    assert torch.equal(ia, ib)
    assert rel_err(a.float().cpu().numpy(), b.float().cpu().numpy()) <= BF16_TOL


@pytest.mark.parametrize("dtype,T", [(torch.float32, 32), (torch.bfloat16, 32), (torch.float32, 1)])
def test_v3_decode_matches_oracle(v3, dtype, T):
    layer, np_exp, np_sh, gw, ocfg = v3
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(50 + T)).to(dtype)
    out, idx, w = layer.forward(x.cuda(), return_routing=True)      # auto: decode GEMVs
    ro, ri, rw = qo.layer_forward(ocfg, gw, np_exp, x.float().numpy(), shared=np_sh,
                                  nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(w.cpu().numpy(), rw)
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert rel_err(out.float().cpu().numpy(), ro) <= tol


def test_v3_zipf_biased_routing_matches_oracle(v3):
    # configs[4]'s router: a per-expert selection bias fitted so expert
    # popularity follows a Zipf(1.1) head (hottest ~8 % of assignments);
    # sampled tokens of a 2048-token batch against the oracle with the same
    # bias, routing bit-exact
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    import bench
    layer0, np_exp, np_sh, gw, ocfg = v3
    W = bench.V3
    bias, target = bench.zipf_bias(W, torch.from_numpy(gw).cuda(), seed=99)
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=IS, scoring=capi.QMOE_SCORING_SIGMOID,
                    n_group=8, topk_group=4, norm_topk_prob=True, routed_scaling_factor=2.5)
    layer = QMoELayer(cfg, gw, np_exp, shared=np_sh, bias=bias.cpu().numpy())
    T = 2048
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(61)).bfloat16()
    out, idx, w = layer.forward(x.cuda(), return_routing=True)
    torch.cuda.synchronize()
    share = np.bincount(idx.cpu().numpy().reshape(-1), minlength=E) / (T * K)
    assert 0.05 <= share.max() <= 0.11, share.max()
    assert int(np.argmax(share)) == int(np.argmax(target))
    sample = np.sort(np.random.default_rng(8).choice(T, 32, replace=False))
    ro, ri, rw = qo.layer_forward(ocfg, gw, np_exp, x[sample].float().numpy(), shared=np_sh,
                                  bias=bias.cpu().numpy(), nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy()[sample], ri)
    np.testing.assert_array_equal(w.cpu().numpy()[sample], rw)
    assert rel_err(out.float().cpu().numpy()[sample], ro) <= BF16_TOL
    layer.close()
