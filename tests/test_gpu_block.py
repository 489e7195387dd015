"""GPU parity of the decoder-layer MoE block (qmoe_layer_forward_block):
out = x + MoE(LN(x)) + Shared(LN(x)) with LN the post-attention LayerNorm
(qmoe-rs src/model.rs:366-367, :400-412), against the oracle's block
(pinned LayerNorm order, then the layer, then the residual add).

Bars: routing bit-exact (the router sees the normalised rows, computed in
the pinned order on both sides; bf16 forwards round them to bf16 on both
sides), outputs within 1e-4 (f32) / 2e-2 (bf16) max-abs relative error."""
import os

import numpy as np
import pytest
import torch

import helpers
from helpers import rel_err
from oracle import oracle as qo
from qmoe_b200 import MoEConfig, QMoELayer, capi

pytestmark = pytest.mark.gpu
NTHREADS = max(1, min(8, os.cpu_count() or 1))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def ln_params(H, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(H, generator=g)).numpy(), (0.05 * torch.randn(H, generator=g)).numpy()


@pytest.mark.parametrize("dtype,T,sigmoid", [(torch.float32, 32, False), (torch.bfloat16, 300, True),
                                             (torch.float32, 1, True), (torch.bfloat16, 64, False)])
def test_block_matches_oracle(dtype, T, sigmoid):
    E, K, H, I, Is = 16, 4, 512, 256, 320
    kw = dict(scoring=capi.QMOE_SCORING_SIGMOID, n_group=4, topk_group=2, norm_topk_prob=True,
              routed_scaling_factor=2.5) if sigmoid else {}
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=Is, **kw)
    experts, shared, gw = helpers.synth_layer(E, H, I, Is, seed=T + 3, device="cuda")
    layer = QMoELayer(cfg, gw, experts, shared=shared)
    w, b = ln_params(H, T)
    layer.set_norm(w, b, 1e-6)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(T)) * 2 + 0.5).to(dtype)
    out, idx, wt = layer.forward_block(x.cuda(), return_routing=True)
    ocfg = qo.MoEConfig(E, K, H, I, Is, scoring=cfg.scoring, n_group=cfg.n_group,
                        topk_group=cfg.topk_group, norm_topk_prob=cfg.norm_topk_prob,
                        routed_scaling_factor=cfg.routed_scaling_factor)
    ref, ri, rw = qo.block_forward(ocfg, gw.cpu().numpy(), helpers.to_numpy_experts(experts),
                                   x.float().numpy(), w, b, 1e-6,
                                   shared=helpers.to_numpy_experts([shared])[0], nthreads=NTHREADS,
                                   round_bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_err(out.float().cpu().numpy(), ref) <= tol
    # host pointers give the device path's bits
    host = layer.forward_block(x)
    assert torch.equal(host, out.cpu())


def test_block_without_experts_adds_the_shared_ffn():
    H, Is = 512, 256
    cfg = MoEConfig(8, 2, H, 128, shared_intermediate_dim=Is)
    _, shared, _ = helpers.synth_layer(1, H, 128, Is, seed=4, device="cuda")
    layer = QMoELayer(cfg, None, [], shared=shared)
    w, b = ln_params(H, 9)
    layer.set_norm(w, b, 1e-5)
    x = torch.randn(20, H, generator=torch.Generator().manual_seed(1))
    out = layer.forward_block(x.cuda()).cpu().numpy()
    y = qo.layernorm(x.numpy(), w, b, 1e-5)
    ref = x.numpy() + qo.shared_forward(helpers.to_numpy_experts([shared])[0], y, H, Is)
    assert rel_err(out, ref) <= 1e-4
    bare = QMoELayer(MoEConfig(8, 2, H, 128), None, [])
    bare.set_norm(w, b)
    assert torch.equal(bare.forward_block(x.cuda()).cpu(), x)


@pytest.mark.parametrize("dtype,T", [(torch.float32, 8), (torch.bfloat16, 256)])
def test_chain_of_blocks_matches_blockwise_and_oracle(dtype, T):
    # the layer loop of forward_next (src/model.rs:481-489) over MoE blocks:
    # the chain's captured graph gives the bits of the blocks called one by
    # one, on every repeat with new inputs in the same buffers
    from qmoe_b200 import BlockChain
    E, K, H, I, Is = 16, 4, 512, 256, 256
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=Is)
    layers, params = [], []
    for l in range(3):
        experts, shared, gw = helpers.synth_layer(E, H, I, Is, seed=50 + l, device="cuda")
        L = QMoELayer(cfg, gw, experts, shared=shared)
        w, b = ln_params(H, 60 + l)
        L.set_norm(w, b)
        layers.append(L)
        params.append((gw.cpu().numpy(), helpers.to_numpy_experts(experts),
                       helpers.to_numpy_experts([shared])[0], w, b))
    chain = BlockChain(layers)
    xbuf = torch.empty(T, H, dtype=dtype, device="cuda")
    obuf = torch.empty(T, H, dtype=dtype, device="cuda")
    with torch.cuda.stream(torch.cuda.Stream()):
        for i in range(3):
            xbuf.copy_(torch.randn(T, H, generator=torch.Generator().manual_seed(70 + i)).to(dtype))
            chain.forward(xbuf, out=obuf)
            ref = xbuf
            for L in layers:
                ref = L.forward_block(ref)
            torch.cuda.synchronize()
            assert torch.equal(obuf, ref), f"call {i}"
    # two blocks against the oracle
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(5)).to(dtype)
    two = BlockChain(layers[:2]).forward(x.cuda())
    y = x.float().numpy()
    for gw, ne, ns, w, b in params[:2]:
        y, _, _ = qo.block_forward(qo.MoEConfig(E, K, H, I, Is), gw, ne, y, w, b, 1e-6, shared=ns,
                                   nthreads=NTHREADS, round_bf16=dtype == torch.bfloat16)
        if dtype == torch.bfloat16:
            y = torch.from_numpy(y).bfloat16().float().numpy()     # the block's bf16 output
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_err(two.float().cpu().numpy(), y) <= tol
    host = BlockChain(layers).forward(x)                           # host pointers
    assert torch.equal(host, chain.forward(x.cuda()).cpu())
