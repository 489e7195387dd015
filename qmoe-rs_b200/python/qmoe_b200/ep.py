"""Expert-parallel MoE layer: the qmoe-rs layer split over the GPUs of a node.

qmoe-rs runs every expert of QMoELayer::forward in one process
(src/moe.rs:40-130).  Here `world` ranks (one process per GPU, torch
distributed over NCCL) each hold `num_experts / world` consecutive experts
and a replica of the gate and the shared expert, and each owns a slice of
the batch.  One forward on every rank:

  1. route its own tokens (qmoe_layer_route: gate, scores, top-k, weights);
  2. plan (qmoe_ep_plan): every token goes once to each rank that owns one
     of its experts, with that rank's local expert ids and weights;
  3. dispatch: all-to-all of the token rows and of their (ids, weights);
  4. run the local experts on what arrived (qmoe_layer_forward_routed): one
     partial sum per received row, over this rank's experts in ascending
     order;
  5. return: all-to-all of the partial rows back to their origin;
  6. combine (qmoe_combine_rows): add each token's partials in ascending
     rank order -- ascending expert blocks, the reference's expert order --
     then add the shared expert's output (qmoe_layer_shared_forward with
     accumulate; src/model.rs:386-389: routed sum first, then + shared).

The exchanges use fixed-size buffers (each destination gets `capacity` rows,
unused rows carry expert ids -1 and are skipped), so a forward needs no
device-to-host read of the counts and can be captured in a CUDA graph.
"""
from __future__ import annotations

try:
    import torch
except ImportError:  # pragma: no cover - the EP layer needs torch.distributed
    torch = None

from . import capi
from .layer import MoEConfig, QMoELayer


class TorchComm:
    """The exchanges of the EP forward over a torch.distributed group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_to_all(self, out, inp):
        """Equal splits along dim 0: out[r-th block] <- rank r's inp[my block]."""
        self.dist.all_to_all_single(out, inp, group=self.group)
        return out


class ExpertParallelMoE:
    """One rank of an expert-parallel layer.

    experts: this rank's experts only (num_experts / world entries, global ids
    rank * experts_per_rank ...).  gate_weight, bias and shared are the full
    replicated tensors.  Inputs and outputs are this rank's tokens [T, H] on
    the rank's GPU, f32 or bf16; `capacity` bounds T per forward.
    """

    def __init__(self, config: MoEConfig, gate_weight, experts, rank: int, world: int,
                 shared=None, bias=None, ctx=None, comm=None, capacity: int = 256):
        if config.num_experts % world:
            raise ValueError(f"num_experts {config.num_experts} not divisible by world {world}")
        if not 1 <= world <= 32:
            raise ValueError("world must be in 1..32")
        self.config = config
        self.rank, self.world = rank, world
        self.epr = config.num_experts // world
        if len(experts) != self.epr:
            raise ValueError(f"expected {self.epr} local experts, got {len(experts)}")
        self.layer = QMoELayer(config, gate_weight, experts, shared=shared, bias=bias, ctx=ctx,
                               expert_begin=rank * self.epr)
        self.has_shared = shared is not None
        self.comm = comm
        self.capacity = int(capacity)
        self._bufs = {}

    # -- device steps (C ABI); split out so tests can exercise the exchanges
    def route(self, x):
        return self.layer.route(x)

    def plan(self, idx, w, T: int):
        G, K, C = self.world, self.config.top_k, self.capacity
        dev = idx.device
        b = self._buf("plan", lambda: dict(
            counts=torch.empty(G, dtype=torch.int32, device=dev),
            tok=torch.empty(G * C, dtype=torch.int32, device=dev),
            ids=torch.empty(G * C, K, dtype=torch.int32, device=dev),
            w=torch.empty(G * C, K, dtype=torch.float32, device=dev),
            slot=torch.empty(C, G, dtype=torch.int32, device=dev)))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_ep_plan", self.layer.ctx.handle, idx.data_ptr(), w.data_ptr(), T, K,
                  self.epr, G, C, b["counts"].data_ptr(), b["tok"].data_ptr(),
                  b["ids"].data_ptr(), b["w"].data_ptr(), b["slot"].data_ptr())
        return b["counts"], b["tok"], b["ids"], b["w"], b["slot"][:T]

    def gather(self, x, tok):
        H = x.shape[1]
        out = self._buf(("gather", x.dtype), lambda: torch.empty(
            self.world * self.capacity, H, dtype=x.dtype, device=x.device))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_gather_rows", self.layer.ctx.handle, x.data_ptr(), _dt(x), H,
                  tok.data_ptr(), tok.numel(), out.data_ptr())
        return out

    def experts(self, rx, rids, rw):
        return self.layer.forward_routed(rx, rids, rw)

    def combine(self, back, slot, T: int, dtype):
        H = back.shape[1]
        out = torch.empty(T, H, dtype=dtype, device=back.device)
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_combine_rows", self.layer.ctx.handle, back.data_ptr(), _dt(back), H,
                  slot.data_ptr(), self.world, T, out.data_ptr())
        return out

    def shared_add(self, x, out):
        if self.has_shared:
            self.layer.shared_forward(x, out=out)
        return out

    # -- forward ------------------------------------------------------------
    def dispatch(self, x):
        """Steps 1-2: route, plan, gather.  Returns (state, rows, meta): the
        send rows [world * capacity, H] and their (local ids, weight bits)
        [world * capacity, 2K] int32, destination d's block at d * capacity."""
        T, H = x.shape
        if T > self.capacity:
            raise ValueError(f"T {T} > capacity {self.capacity}")
        idx, w = self.route(x)
        counts, tok, ids, wts, slot = self.plan(idx, w, T)
        rows = self.gather(x, tok)
        meta = torch.cat([ids, wts.view(torch.int32)], dim=1)
        return (x, slot, idx, w), rows, meta

    def compute(self, rows, meta):
        """Step 4: this rank's experts on the received rows (block r from rank
        r), one partial row per received row."""
        K = self.config.top_k
        rids = meta[:, :K].contiguous()
        rw = meta[:, K:].contiguous().view(torch.float32)
        return self.experts(rows, rids, rw)

    def finish(self, state, back):
        """Step 6: add each token's returned partials in ascending rank order,
        then the shared expert."""
        x, slot, _, _ = state
        out = self.combine(back, slot, x.shape[0], x.dtype)
        return self.shared_add(x, out)

    def forward(self, x, return_routing: bool = False):
        if self.comm is None:
            self.comm = TorchComm()
        state, rows, meta = self.dispatch(x)
        rx = self._buf(("rx", rows.dtype), lambda: torch.empty_like(rows))
        rmeta = self._buf("rmeta", lambda: torch.empty_like(meta))
        self.comm.all_to_all(rx, rows)
        self.comm.all_to_all(rmeta, meta)
        y = self.compute(rx, rmeta)
        back = self._buf(("back", y.dtype), lambda: torch.empty_like(y))
        self.comm.all_to_all(back, y)
        out = self.finish(state, back)
        if return_routing:
            return out, state[2], state[3]
        return out

    def _buf(self, key, make):
        b = self._bufs.get(key)
        if b is None:
            b = make()
            self._bufs[key] = b
        return b


def _dt(t) -> int:
    return capi.QMOE_DTYPE_BF16 if t.dtype == torch.bfloat16 else capi.QMOE_DTYPE_F32
