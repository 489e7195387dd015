"""CPU checks of the benchmark's workload generators and of its two arms'
agreement on the measured configuration (no GPU involved)."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_zipf_targets_shape():
    p = bench.zipf_targets(256)
    assert abs(p.sum() - 1.0) < 1e-12
    assert abs(p[0] - 0.08) < 1e-6                       # the hottest expert's share
    assert np.all(np.diff(p) < 0)
    # the tail follows (r + q)^-1.1: successive ratios approach (r / (r+1))^1.1
    r = np.arange(200, 255)
    ratio = p[r + 1] / p[r]
    assert np.all(ratio < 1.0) and np.all(ratio > (r / (r + 1.0)) ** 1.1)


def test_zipf_bias_gives_a_hot_head():
    # a V3-style router (sigmoid, 8 groups, top-4 groups, top-8) on a smaller
    # hidden size: the fitted bias puts ~8 % of the assignments on the
    # hottest expert of the seeded permutation, and the shares fall off
    W = dict(bench.V3, H=512)
    g = torch.Generator().manual_seed(3)
    gate = torch.randn(W["E"], W["H"], generator=g) * 0.02
    bias, target = bench.zipf_bias(W, gate, seed=11, tokens=2048, iters=200)
    x = torch.randn(4096, W["H"], generator=torch.Generator().manual_seed(12))
    idx = bench.route_torch(W, x @ gate.t(), bias)
    share = torch.bincount(idx.reshape(-1), minlength=W["E"]).double() / idx.numel()
    order = np.argsort(-target)
    head = share.numpy()[order[:4]]
    assert 0.06 <= head[0] <= 0.10, head
    assert head[0] > head[3]
    assert bias.shape == (W["E"],) and torch.isfinite(bias).all()


def test_both_arms_print_the_same_config():
    class A:
        pass
    for W in (bench.V3, bench.V2):
        for n in (1, 2, 8):
            assert bench.headline_config(W, n, A()) == bench.headline_config(W, n, A())
    c = bench.headline_config(bench.V3, 8, A())
    assert c["T_per_gpu"] == 4096 and c["experts_per_gpu"] == 32 and c["parallelism"] == "ep8"


def test_algorithmic_counts():
    W = bench.V3
    gu, dn, total = bench.layer_flops(W, 4096)
    assert gu == 2.0 * 4096 * 8 * 2 * 7168 * 2048 + 2.0 * 4096 * 2 * 7168 * 2048
    assert abs(total - 3.262e12) / 3.262e12 < 1e-3       # the survey's 3.26e12 FLOP
    assert bench.per_expert_bytes(W) == 11055104          # 3 H I / 4 + 4 (2 I + H)
