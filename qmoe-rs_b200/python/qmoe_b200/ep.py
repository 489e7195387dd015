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
  4. run the local experts on what arrived, and the shared expert on the
     rank's own tokens appended after them, in one pass
     (qmoe_layer_forward_ep): one partial sum per received row, over this
     rank's experts in ascending order;
  5. return: all-to-all of the partial rows back to their origin;
  6. combine (qmoe_combine_rows): add each token's partials in ascending
     rank order -- ascending expert blocks, the reference's expert order --
     then the shared expert's row (src/model.rs:386-389: routed sum first,
     then + shared).

The exchanges use fixed-size buffers (each destination gets `capacity` rows,
unused rows carry expert ids -1 and are skipped), so a forward needs no
device-to-host read of the counts and can be captured in a CUDA graph.

Two ways to move the rows: `exchange="nccl"` (all-to-alls over the process
group) or `exchange="p2p"` (PeerExchange: steps 3 and 5 as kernels that store
straight into the other GPUs' memory over NVLink, each followed by a bounded
wait on the peers' arrival flags).
"""
from __future__ import annotations

try:
    import torch
except ImportError:  # pragma: no cover - the EP layer needs torch.distributed
    torch = None

import ctypes

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


class PeerExchange:
    """One rank's exchange buffers in peer memory (qmoe_ep_peer_*): receive
    rows and metadata, returned rows, arrival flags; the ranks open each
    other's buffers through CUDA IPC handles gathered over `group`."""

    def __init__(self, ctx, world: int, rank: int, capacity: int, H: int, K: int, dtype_code: int,
                 group=None):
        import torch.distributed as dist
        h = ctypes.c_void_p()
        capi.call("qmoe_ep_peer_create", ctx.handle, world, rank, capacity, H, K, dtype_code,
                  ctypes.byref(h))
        self._h = h
        mine = (ctypes.c_uint8 * capi.QMOE_EP_HANDLE_BYTES)()
        capi.call("qmoe_ep_peer_handle", h, mine)
        dev = torch.device("cuda", ctx.device)
        t = torch.tensor(list(bytes(mine)), dtype=torch.uint8, device=dev)
        allh = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allh, t, group=group)
        blob = bytes(torch.cat(allh).cpu().tolist())
        buf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        capi.call("qmoe_ep_peer_connect", h, buf)
        dist.barrier(group=group)
        rows, meta, back = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        capi.call("qmoe_ep_peer_buffers", h, ctypes.byref(rows), ctypes.byref(meta), ctypes.byref(back))
        self.recv_rows, self.recv_meta, self.back_rows = rows.value, meta.value, back.value

    def dispatch(self, x, T: int, counts, tok, meta):
        capi.call("qmoe_ep_dispatch", self._h, ctypes.c_void_p(x.data_ptr()), T,
                  ctypes.c_void_p(counts.data_ptr()), ctypes.c_void_p(tok.data_ptr()),
                  ctypes.c_void_p(meta.data_ptr()))

    def wait(self, phase: int):
        capi.call("qmoe_ep_wait", self._h, phase)

    def give_back(self, y):
        capi.call("qmoe_ep_return", self._h, ctypes.c_void_p(y.data_ptr()))

    def finish(self, slot, T: int, extra, out):
        """Wait for every peer's returned rows, then out[t] = the sum of t's
        returned partials in rank order + extra[t] (one launch)."""
        capi.call("qmoe_ep_finish", self._h, slot.data_ptr(), T,
                  extra.data_ptr() if extra is not None else None, out.data_ptr())

    def close(self):
        if getattr(self, "_h", None):
            capi.lib().qmoe_ep_peer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertParallelMoE:
    """One rank of an expert-parallel layer.

    experts: this rank's experts only (num_experts / world entries, global ids
    rank * experts_per_rank ...).  gate_weight, bias and shared are the full
    replicated tensors.  Inputs and outputs are this rank's tokens [T, H] on
    the rank's GPU, f32 or bf16; `capacity` bounds T per forward.
    """

    def __init__(self, config: MoEConfig, gate_weight, experts, rank: int, world: int,
                 shared=None, bias=None, ctx=None, comm=None, capacity: int = 256,
                 exchange: str = "nccl", dtype=None, group=None):
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
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', not {exchange!r}")
        self.exchange = exchange
        self.peer = None
        if exchange == "p2p":
            dt = capi.QMOE_DTYPE_BF16 if dtype == torch.bfloat16 else capi.QMOE_DTYPE_F32
            self.dtype = torch.bfloat16 if dt == capi.QMOE_DTYPE_BF16 else torch.float32
            self.peer = PeerExchange(self.layer.ctx, world, rank, self.capacity,
                                     config.hidden_dim, config.top_k, dt, group=group)

    # -- device steps (C ABI); split out so tests can exercise the exchanges
    def route(self, x):
        return self.layer.route(x)

    def plan(self, idx, w, T: int):
        """Send list: counts [G], tokens [G*C], meta [G*C, 2K] (local ids, then
        weight bits), slot [T, G] (send row of (token, rank))."""
        G, K, C = self.world, self.config.top_k, self.capacity
        dev = idx.device
        b = self._buf("plan", lambda: dict(
            counts=torch.empty(G, dtype=torch.int32, device=dev),
            tok=torch.empty(G * C, dtype=torch.int32, device=dev),
            meta=torch.empty(G * C, 2 * K, dtype=torch.int32, device=dev),
            slot=torch.empty(C, G, dtype=torch.int32, device=dev)))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_ep_plan", self.layer.ctx.handle, idx.data_ptr(), w.data_ptr(), T, K,
                  self.epr, G, C, b["counts"].data_ptr(), b["tok"].data_ptr(),
                  b["meta"].data_ptr(), b["slot"].data_ptr())
        return b["counts"], b["tok"], b["meta"], b["slot"][:T]

    def route_plan(self, x):
        """route() then plan() on this rank's tokens in one C-ABI call (one
        kernel launch for decode-sized batches) -> (idx, w, counts, tok,
        meta, slot)."""
        T = x.shape[0]
        G, K, C = self.world, self.config.top_k, self.capacity
        dev = x.device
        b = self._buf("plan", lambda: dict(
            counts=torch.empty(G, dtype=torch.int32, device=dev),
            tok=torch.empty(G * C, dtype=torch.int32, device=dev),
            meta=torch.empty(G * C, 2 * K, dtype=torch.int32, device=dev),
            slot=torch.empty(C, G, dtype=torch.int32, device=dev)))
        r = self._buf("routing", lambda: dict(
            idx=torch.empty(C, K, dtype=torch.int32, device=dev),
            w=torch.empty(C, K, dtype=torch.float32, device=dev)))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_route_plan", self.layer._h, x.data_ptr(), _dt(x), T,
                  r["idx"].data_ptr(), r["w"].data_ptr(), self.epr, G, C, b["counts"].data_ptr(),
                  b["tok"].data_ptr(), b["meta"].data_ptr(), b["slot"].data_ptr())
        return r["idx"][:T], r["w"][:T], b["counts"], b["tok"], b["meta"], b["slot"][:T]

    def gather(self, x, tok):
        H = x.shape[1]
        out = self._buf(("gather", x.dtype), lambda: torch.empty(
            self.world * self.capacity, H, dtype=x.dtype, device=x.device))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_gather_rows", self.layer.ctx.handle, x.data_ptr(), _dt(x), H,
                  tok.data_ptr(), tok.numel(), out.data_ptr())
        return out

    def run_rows(self, rows, meta, R: int, shared_row0: int):
        """Local experts over rows[:R] (routing in meta) + the shared expert
        over rows shared_row0..R-1."""
        H = rows.shape[1]
        y = self._buf(("y", rows.dtype), lambda: torch.empty(rows.shape[0], H, dtype=rows.dtype,
                                                              device=rows.device))
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_forward_ep", self.layer._h, rows.data_ptr(), _dt(rows), R,
                  meta.data_ptr(), shared_row0, y.data_ptr())
        return y

    def combine(self, back, slot, extra, T: int, dtype):
        H = back.shape[1]
        out = torch.empty(T, H, dtype=dtype, device=back.device)
        self.layer.ctx.use_current_torch_stream()
        capi.call("qmoe_combine_rows", self.layer.ctx.handle, back.data_ptr(), _dt(back), H,
                  slot.data_ptr(), self.world, T,
                  extra.data_ptr() if extra is not None else None, out.data_ptr())
        return out

    # -- forward ------------------------------------------------------------
    def dispatch(self, x):
        """Steps 1-2: route, plan, gather.  Returns (state, rows, meta): the
        send rows [world * capacity, H] and their meta [world * capacity, 2K]
        int32, destination d's block at d * capacity."""
        T, H = x.shape
        if T > self.capacity:
            raise ValueError(f"T {T} > capacity {self.capacity}")
        idx, w = self.route(x)
        counts, tok, meta, slot = self.plan(idx, w, T)
        rows = self.gather(x, tok)
        return (x, slot, idx, w), rows, meta

    def recv_buffers(self, x):
        """Receive rows [world*C + C, H] and meta [world*C + C, 2K]: the first
        world*C rows are the all-to-all targets, the last C rows take this
        rank's own tokens for the shared expert (their expert ids stay -1)."""
        G, C, K = self.world, self.capacity, self.config.top_k
        H = x.shape[1]
        rx = self._buf(("rx", x.dtype), lambda: torch.empty(G * C + C, H, dtype=x.dtype,
                                                              device=x.device))

        def make_meta():
            m = torch.zeros(G * C + C, 2 * K, dtype=torch.int32, device=x.device)
            m[:, :K] = -1
            return m
        return rx, self._buf("rmeta", make_meta)

    def compute(self, rx, rmeta, x):
        """Step 4: this rank's experts on the received rows rx[:world*C]
        (block r from rank r) and the shared expert on its own tokens x.
        Returns y: rows [:world*C] the partials to return, rows
        [world*C : world*C + T] the shared expert's output for x."""
        GC, T = self.world * self.capacity, x.shape[0]
        if self.has_shared:
            rx[GC:GC + T].copy_(x)
            return self.run_rows(rx, rmeta, GC + T, GC)
        return self.run_rows(rx, rmeta, GC, GC)

    def finish(self, state, back, y):
        """Step 6: each token's returned partials in ascending rank order, then
        the shared expert's row."""
        x, slot, _, _ = state
        GC, T = self.world * self.capacity, x.shape[0]
        extra = y[GC:GC + T] if self.has_shared else None
        return self.combine(back, slot, extra, T, x.dtype)

    def forward_p2p(self, x, return_routing: bool = False):
        """The forward with the exchanges over peer memory: route and send
        list (one kernel for decode batches), dispatch kernel, this rank's
        experts on the received rows and the shared expert on its own tokens
        (the first kernel waits for the peers' rows, the last returns the
        partial sums to their ranks), finish (wait for the returns, combine)."""
        if x.dtype != self.dtype:
            raise TypeError(f"this exchange carries {self.dtype} rows, got {x.dtype}")
        T, H = x.shape
        if T > self.capacity:
            raise ValueError(f"T {T} > capacity {self.capacity}")
        G, C, K = self.world, self.capacity, self.config.top_k
        GC = G * C
        idx, w, counts, tok, meta, slot = self.route_plan(x)
        ctx = self.layer.ctx
        ctx.use_current_torch_stream()
        self.peer.dispatch(x, T, counts, tok, meta)
        y = self._buf(("y", x.dtype), lambda: torch.empty(GC + C, H, dtype=x.dtype, device=x.device))
        R = GC + T if self.has_shared else GC
        # the expert pass waits for the peers' rows in its first kernel and
        # stores the received rows' partial sums straight into their origin
        # ranks' return blocks (or runs the return kernel)
        capi.call("qmoe_layer_forward_ep_return", self.layer._h, self.peer._h,
                  ctypes.c_void_p(self.peer.recv_rows), _dt(x), R, ctypes.c_void_p(self.peer.recv_meta),
                  GC, y.data_ptr())
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
        extra = y[GC:GC + T] if self.has_shared else None
        self.peer.finish(slot, T, extra, out)
        if return_routing:
            return out, idx.clone(), w.clone()
        return out

    def forward(self, x, return_routing: bool = False):
        if getattr(self, "peer", None) is not None:
            return self.forward_p2p(x, return_routing)
        if self.comm is None:
            self.comm = TorchComm()
        GC = self.world * self.capacity
        state, rows, meta = self.dispatch(x)
        rx, rmeta = self.recv_buffers(x)
        self.comm.all_to_all(rx[:GC], rows)
        self.comm.all_to_all(rmeta[:GC], meta)
        y = self.compute(rx, rmeta, x)
        back = self._buf(("back", y.dtype), lambda: torch.empty(GC, y.shape[1], dtype=y.dtype,
                                                                device=y.device))
        self.comm.all_to_all(back, y[:GC])
        out = self.finish(state, back, y)
        if return_routing:
            return out, state[2], state[3]
        return out

    def close(self):
        if getattr(self, "peer", None) is not None:
            self.peer.close()
            self.peer = None

    def _buf(self, key, make):
        b = self._bufs.get(key)
        if b is None:
            b = make()
            self._bufs[key] = b
        return b


def _dt(t) -> int:
    return capi.QMOE_DTYPE_BF16 if t.dtype == torch.bfloat16 else capi.QMOE_DTYPE_F32
