"""Expert-parallel exchange logic on CPU: two gloo ranks, device steps
replaced by the oracle (HostRank), output against the single-process
oracle layer.  Covers the host orchestration of ExpertParallelMoE (plan
layout, the three all-to-alls, the return map, ascending-rank combine, the
shared expert added last) without a GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import helpers
from ep_ref import HostRank
from oracle import oracle as qo
from qmoe_b200 import MoEConfig, TorchComm

E, K, H, I, IS, T_RANK = 8, 3, 64, 64, 128, 10


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer():
    experts, shared, gate_w = helpers.synth_layer(E, H, I, IS, seed=21)
    return (helpers.to_numpy_experts(experts), helpers.to_numpy_experts([shared])[0],
            gate_w.numpy())


def _worker(rank, world, port, capacity, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        experts, shared, gate_w = _layer()
        cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=IS)
        qcfg = qo.MoEConfig(E, K, H, I, IS)
        x = torch.from_numpy(np.random.default_rng(7).standard_normal(
            (world * T_RANK, H)).astype(np.float32))
        mine = x[rank * T_RANK:(rank + 1) * T_RANK]
        ep = HostRank(cfg, qcfg, gate_w, experts, shared, rank, world, TorchComm(), capacity)
        out, idx, _ = ep.forward(mine, return_routing=True)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(out_dir, f"idx{rank}.npy"), idx.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,capacity", [(2, T_RANK), (2, 16), (4, T_RANK)])
def test_ep_exchange_matches_single_process(tmp_path, world, capacity):
    mp.spawn(_worker, args=(world, _free_port(), capacity, str(tmp_path)), nprocs=world, join=True)
    experts, shared, gate_w = _layer()
    x = np.random.default_rng(7).standard_normal((world * T_RANK, H)).astype(np.float32)
    ro, ri, _ = qo.layer_forward(qo.MoEConfig(E, K, H, I, IS), gate_w, experts, x, shared=shared)
    out = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(world)])
    idx = np.concatenate([np.load(tmp_path / f"idx{r}.npy") for r in range(world)])
    np.testing.assert_array_equal(idx, ri)
    assert helpers.rel_err(out, ro) <= 1e-5


def test_plan_reference_layouts():
    from ep_ref import plan_reference
    idx = np.array([[0, 5], [2, 3], [7, -1], [1, 6]], np.int32)
    w = np.arange(8, dtype=np.float32).reshape(4, 2)
    # experts 2 per rank: token destinations {0,2}, {1}, {3}, {0,3}
    c, tok, ids, ww, slot = plan_reference(idx, w, 2, 4, 0)
    np.testing.assert_array_equal(c, [2, 1, 1, 2])
    np.testing.assert_array_equal(tok[:6], [0, 3, 1, 0, 2, 3])
    np.testing.assert_array_equal(slot, [[0, -1, 3, -1], [-1, 2, -1, -1], [-1, -1, -1, 4],
                                         [1, -1, -1, 5]])
    np.testing.assert_array_equal(ids[:4], [[0, -1], [1, -1], [0, 1], [-1, 1]])
    np.testing.assert_array_equal(ww[:4], [[0, 0], [6, 0], [2, 3], [0, 1]])
    c2, tok2, ids2, ww2, slot2 = plan_reference(idx, w, 2, 4, 5)
    np.testing.assert_array_equal(c2, c)
    np.testing.assert_array_equal(slot2, [[0, -1, 10, -1], [-1, 5, -1, -1], [-1, -1, -1, 15],
                                          [1, -1, -1, 16]])
    assert (ids2[2:5] == -1).all() and (ww2[2:5] == 0).all() and (tok2[2:5] == 0).all()
