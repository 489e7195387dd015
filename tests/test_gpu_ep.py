"""Expert-parallel layer on one GPU: the device steps of every rank
(qmoe_ep_plan, qmoe_gather_rows, forward_routed on a rank's expert block,
qmoe_combine_rows, shared add) run for G virtual ranks; the all-to-alls are
done by slicing.  Outputs against the single-process oracle layer."""
import os

import numpy as np
import pytest
import torch

import helpers
from ep_ref import plan_reference
from helpers import rel_err
from oracle import oracle as qo
from qmoe_b200 import ExpertParallelMoE, MoEConfig, capi

pytestmark = pytest.mark.gpu
NTHREADS = max(1, min(8, os.cpu_count() or 1))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def exchange(blocks, G, C):
    """all-to-all with equal splits: rank r receives block r of every rank."""
    return [torch.cat([blocks[s][r * C:(r + 1) * C] for s in range(G)]) for r in range(G)]


def run_virtual(ranks, xs, G, C):
    st, rows, metas = zip(*[rk.dispatch(x) for rk, x in zip(ranks, xs)])
    rx, rm = exchange(rows, G, C), exchange(metas, G, C)
    ys = []
    for rk, a, b, x in zip(ranks, rx, rm, xs):
        rbuf, mbuf = rk.recv_buffers(x)
        rbuf[:G * C].copy_(a)
        mbuf[:G * C].copy_(b)
        ys.append(rk.compute(rbuf, mbuf, x).clone())
    back = exchange([y[:G * C] for y in ys], G, C)
    outs = [rk.finish(s, b, y) for rk, s, b, y in zip(ranks, st, back, ys)]
    idx = torch.cat([s[2] for s in st])
    return torch.cat(outs), idx


@pytest.mark.parametrize("G,dtype,scoring", [
    (2, torch.float32, capi.QMOE_SCORING_SOFTMAX),
    (4, torch.float32, capi.QMOE_SCORING_SIGMOID),
    (8, torch.bfloat16, capi.QMOE_SCORING_SOFTMAX),
])
def test_ep_virtual_ranks_match_oracle(G, dtype, scoring):
    E, K, H, I, Is, Tr = 16, 4, 256, 128, 192, 9
    kw = dict(scoring=scoring)
    if scoring == capi.QMOE_SCORING_SIGMOID:
        kw.update(n_group=4, topk_group=2, norm_topk_prob=True, routed_scaling_factor=2.5)
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=Is, **kw)
    experts, shared, gw = helpers.synth_layer(E, H, I, Is, seed=G * 10 + 1, device="cuda")
    epr = E // G
    ranks = [ExpertParallelMoE(cfg, gw, experts[r * epr:(r + 1) * epr], r, G, shared=shared,
                               capacity=16) for r in range(G)]
    x = torch.randn(G * Tr, H, generator=torch.Generator().manual_seed(G))
    if dtype == torch.bfloat16:
        x = x.bfloat16()
    xs = [x[r * Tr:(r + 1) * Tr].cuda() for r in range(G)]
    out, idx = run_virtual(ranks, xs, G, 16)
    qcfg = qo.MoEConfig(E, K, H, I, Is, cfg.scoring, cfg.n_group, cfg.topk_group,
                        cfg.norm_topk_prob, cfg.routed_scaling_factor)
    ro, ri, _ = qo.layer_forward(qcfg, gw.cpu().numpy(), helpers.to_numpy_experts(experts),
                                 x.float().numpy(), shared=helpers.to_numpy_experts([shared])[0],
                                 nthreads=NTHREADS)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    assert rel_err(out.float().cpu().numpy(), ro) <= tol


@pytest.mark.parametrize("capacity", [0, 40])
def test_ep_plan_kernel_matches_reference(capacity):
    rng = np.random.default_rng(3)
    T, K, epr, G = 37, 6, 8, 8
    idx = np.stack([rng.choice(epr * G, K, replace=False) for _ in range(T)]).astype(np.int32)
    idx[rng.random((T, K)) < 0.1] = -1          # slots skipped
    w = rng.random((T, K), dtype=np.float32)
    from qmoe_b200 import default_context
    ctx = default_context(0)
    rows = G * capacity if capacity else T * G
    dev = "cuda"
    counts = torch.empty(G, dtype=torch.int32, device=dev)
    tok = torch.full((rows,), 7777, dtype=torch.int32, device=dev)
    meta = torch.full((rows, 2 * K), 7777, dtype=torch.int32, device=dev)
    slot = torch.empty(T, G, dtype=torch.int32, device=dev)
    ti, tw = torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda()
    ctx.use_current_torch_stream()
    capi.call("qmoe_ep_plan", ctx.handle, ti.data_ptr(), tw.data_ptr(), T, K, epr, G, capacity,
              counts.data_ptr(), tok.data_ptr(), meta.data_ptr(), slot.data_ptr())
    torch.cuda.synchronize()
    c, rtok, rids, rww, rslot = plan_reference(idx, w, epr, G, capacity)
    np.testing.assert_array_equal(counts.cpu().numpy(), c)
    np.testing.assert_array_equal(slot.cpu().numpy(), rslot)
    m = meta.cpu().numpy()
    ids, ww = m[:, :K], np.ascontiguousarray(m[:, K:]).view(np.float32)
    valid = rslot[rslot >= 0]
    np.testing.assert_array_equal(tok.cpu().numpy()[valid], rtok[valid])
    np.testing.assert_array_equal(ids[valid], rids[valid])
    np.testing.assert_array_equal(ww[valid], rww[valid])
    if capacity:                                 # padded rows: ids -1, weight 0, token 0
        np.testing.assert_array_equal(ids, rids)
        np.testing.assert_array_equal(ww, rww)
        np.testing.assert_array_equal(tok.cpu().numpy(), rtok)


def test_gather_and_combine_rows():
    from qmoe_b200 import default_context
    ctx = default_context(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    for dt, code in ((torch.float32, capi.QMOE_DTYPE_F32), (torch.bfloat16, capi.QMOE_DTYPE_BF16)):
        x = torch.randn(11, 64, generator=g, device="cuda").to(dt)
        idx = torch.tensor([3, 0, 10, 3, 7], dtype=torch.int32, device="cuda")
        out = torch.empty(5, 64, dtype=dt, device="cuda")
        ctx.use_current_torch_stream()
        capi.call("qmoe_gather_rows", ctx.handle, x.data_ptr(), code, 64, idx.data_ptr(), 5,
                  out.data_ptr())
        assert torch.equal(out, x[idx.long()])
        slot = torch.tensor([[0, -1, 4], [-1, -1, -1], [2, 1, 3]], dtype=torch.int32, device="cuda")
        res = torch.empty(3, 64, dtype=dt, device="cuda")
        capi.call("qmoe_combine_rows", ctx.handle, x.data_ptr(), code, 64, slot.data_ptr(), 3, 3,
                  None, res.data_ptr())
        xf = x.float()
        ref = torch.stack([xf[0] + xf[4], torch.zeros(64, device="cuda"), (xf[2] + xf[1]) + xf[3]])
        assert torch.equal(res, ref.to(dt))
        extra = x[8:11].contiguous()
        capi.call("qmoe_combine_rows", ctx.handle, x.data_ptr(), code, 64, slot.data_ptr(), 3, 3,
                  extra.data_ptr(), res.data_ptr())
        assert torch.equal(res, (ref + extra.float()).to(dt))


@pytest.mark.parametrize("G,T,dtype", [
    (2, 1, torch.float32), (2, 33, torch.bfloat16), (8, 64, torch.float32), (4, 100, torch.float32),
])
def test_route_plan_matches_route_then_plan(G, T, dtype):
    """qmoe_layer_route_plan (the front cluster building the send list for
    T <= 64, the router and plan kernels otherwise) against qmoe_layer_route
    followed by qmoe_ep_plan: routing and every send-list array bit-exact."""
    E, K, H, I = 64, 6, 512, 128
    cfg = MoEConfig(E, K, H, I)
    experts, _, gw = helpers.synth_layer(E, H, I, 0, seed=T + G, device="cuda")
    epr = E // G
    C = 128
    rank = ExpertParallelMoE(cfg, gw, experts[:epr], 0, G, capacity=C)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(dtype).cuda()
    idx, w, counts, tok, meta, slot = [a.clone() for a in rank.route_plan(x)]
    ri, rw = rank.route(x)
    rc, rt, rm, rs = rank.plan(ri, rw, T)
    torch.cuda.synchronize()
    for a, b in [(idx, ri), (w, rw), (counts, rc), (tok, rt), (meta, rm), (slot, rs)]:
        assert a.shape == b.shape
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
