"""Host restatement of the expert-parallel plan (test reference for
qmoe_ep_plan) and a CPU stand-in of one EP rank whose device steps run the
oracle, so the exchange logic can be tested on gloo without a GPU."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as qo
from qmoe_b200.ep import ExpertParallelMoE


def plan_reference(idx: np.ndarray, w: np.ndarray, epr: int, world: int, capacity: int):
    """Send list of one rank: destination-major, token order within a
    destination; capacity 0 = compact rows, else rank d's rows at d*capacity
    (unused rows: token 0, ids -1, weight 0)."""
    T, K = idx.shape
    dest = np.where(idx >= 0, idx // epr, -1)
    sends = np.zeros((T, world), bool)
    for t in range(T):
        for k in range(K):
            if dest[t, k] >= 0:
                sends[t, dest[t, k]] = True
    counts = sends.sum(0).astype(np.int32)
    rows = world * capacity if capacity else T * world
    tok = np.zeros(rows, np.int32)
    ids = np.full((rows, K), -1, np.int32)
    ww = np.zeros((rows, K), np.float32)
    slot = np.full((T, world), -1, np.int32)
    base = 0
    for d in range(world):
        r0 = d * capacity if capacity else base
        j = 0
        for t in range(T):
            if not sends[t, d]:
                continue
            r = r0 + j
            j += 1
            tok[r] = t
            mine = dest[t] == d
            ids[r] = np.where(mine, idx[t] - d * epr, -1)
            ww[r] = np.where(mine, w[t], 0.0)
            slot[t, d] = r
        base += counts[d]
    return counts, tok, ids, ww, slot


class HostRank(ExpertParallelMoE):
    """One EP rank whose device steps are the CPU oracle (test stand-in)."""

    def __init__(self, cfg, qcfg, gate_w, experts_np, shared_np, rank, world, comm, capacity):
        self.config = cfg
        self.qcfg = qcfg
        self.rank, self.world = rank, world
        self.epr = cfg.num_experts // world
        self.gate_w = gate_w
        self.local = experts_np[rank * self.epr:(rank + 1) * self.epr]
        self.shared_np = shared_np
        self.has_shared = shared_np is not None
        self.comm = comm
        self.capacity = capacity
        self._bufs = {}

    def route(self, x):
        logits = qo.gate_logits(x.numpy(), self.gate_w)
        idx, w = qo.route(self.qcfg, logits)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def plan(self, idx, w, T):
        c, tok, ids, ww, slot = plan_reference(idx.numpy(), w.numpy(), self.epr, self.world,
                                               self.capacity)
        meta = np.concatenate([ids, ww.view(np.int32)], axis=1)
        return (torch.from_numpy(c), torch.from_numpy(tok), torch.from_numpy(meta),
                torch.from_numpy(slot))

    def gather(self, x, tok):
        return x[tok.long()].clone()

    def run_rows(self, rows, meta, R, shared_row0):
        K = self.config.top_k
        m = meta.numpy()
        ids = np.ascontiguousarray(m[:R, :K])
        ww = np.ascontiguousarray(m[:R, K:]).view(np.float32)
        cfg = qo.MoEConfig(self.epr, K, self.config.hidden_dim, self.config.intermediate_dim)
        y = np.zeros((rows.shape[0], rows.shape[1]), np.float32)
        y[:R] = qo.experts_forward(cfg, self.local, rows[:R].numpy(), ids, ww)
        if self.has_shared and shared_row0 < R:
            sh = qo.shared_forward(self.shared_np, rows[shared_row0:R].numpy(),
                                   self.config.hidden_dim, self.config.shared_intermediate_dim)
            y[shared_row0:R] = y[shared_row0:R] + np.asarray(sh, np.float32)
        return torch.from_numpy(y)

    def combine(self, back, slot, extra, T, dtype):
        b = back.numpy()
        s = slot.numpy()
        out = np.zeros((T, b.shape[1]), np.float32)
        for t in range(T):
            acc = np.zeros(b.shape[1], np.float32)
            for d in range(s.shape[1]):
                if s[t, d] >= 0:
                    acc = acc + b[s[t, d]]
            if extra is not None:
                acc = acc + extra[t].numpy()
            out[t] = acc
        return torch.from_numpy(out)
