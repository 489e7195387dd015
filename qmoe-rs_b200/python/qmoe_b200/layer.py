"""Host-side mirror of qmoe-rs's MoE API over the C ABI.

The classes keep qmoe-rs's names and method contracts so code written
against the Rust crate reads the same here:

  PackedQMoETensor   src/tensor.rs:16-121   from_bytes, shape, scales,
                                            forward_simd, forward_simd_raw
  MoEConfig          src/moe.rs:6-11        (+ routing extensions)
  PackedExpert       src/moe.rs:15-19
  QMoELayer          src/moe.rs:23-130      new / forward, plus the layer's
                     src/model.rs:318-348   SharedExpert (shared_forward)

Every call goes through lib/libqmoe_b200.so.  Inputs may be numpy arrays,
CPU torch tensors (host pointers; copies happen inside the call) or CUDA
torch tensors (device pointers; the call is asynchronous on the current
torch stream).  Outputs come back in the same kind of container.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import capi

try:
    import torch
except ImportError:  # pragma: no cover - torch is part of the image
    torch = None


# ---------------------------------------------------------------------------
# buffers
# ---------------------------------------------------------------------------

def _is_cuda(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor) and x.is_cuda


def _ptr(x):
    """(pointer, ptr_kind, keepalive) for a numpy array or torch tensor."""
    if torch is not None and isinstance(x, torch.Tensor):
        x = x.contiguous()
        kind = capi.QMOE_PTR_DEVICE if x.is_cuda else capi.QMOE_PTR_HOST
        return ctypes.c_void_p(x.data_ptr()), kind, x
    a = np.ascontiguousarray(x)
    return ctypes.c_void_p(a.ctypes.data), capi.QMOE_PTR_HOST, a


def _dtype_code(x) -> int:
    if torch is not None and isinstance(x, torch.Tensor):
        if x.dtype == torch.float32:
            return capi.QMOE_DTYPE_F32
        if x.dtype == torch.bfloat16:
            return capi.QMOE_DTYPE_BF16
        raise TypeError(f"activations must be float32 or bfloat16, got {x.dtype}")
    if np.asarray(x).dtype == np.float32:
        return capi.QMOE_DTYPE_F32
    raise TypeError("numpy activations must be float32")


def _empty_like_kind(x, shape, dtype_code):
    if torch is not None and isinstance(x, torch.Tensor):
        dt = torch.float32 if dtype_code == capi.QMOE_DTYPE_F32 else torch.bfloat16
        return torch.empty(shape, dtype=dt, device=x.device)
    return np.empty(shape, np.float32)


def _empty_aux(x, shape, np_dtype, torch_dtype):
    if torch is not None and isinstance(x, torch.Tensor):
        return torch.empty(shape, dtype=torch_dtype, device=x.device)
    return np.empty(shape, np_dtype)


# ---------------------------------------------------------------------------
# context
# ---------------------------------------------------------------------------

class Context:
    """A device + stream binding (qmoe_ctx)."""

    def __init__(self, device: int = 0, stream: Optional[int] = None):
        h = ctypes.c_void_p()
        capi.call("qmoe_ctx_create", int(device), ctypes.c_void_p(stream or 0), ctypes.byref(h))
        self.handle = h
        self.device = int(device)

    def use_stream(self, stream: Optional[int]) -> None:
        capi.call("qmoe_ctx_set_stream", self.handle, ctypes.c_void_p(stream or 0))

    def use_current_torch_stream(self) -> None:
        if torch is not None and torch.cuda.is_available():
            self.use_stream(torch.cuda.current_stream(self.device).cuda_stream)

    def synchronize(self) -> None:
        capi.call("qmoe_ctx_synchronize", self.handle)

    def close(self) -> None:
        if getattr(self, "handle", None):
            capi.lib().qmoe_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx: dict = {}


def default_context(device: int = 0) -> Context:
    if device not in _default_ctx:
        _default_ctx[device] = Context(device)
    return _default_ctx[device]


# ---------------------------------------------------------------------------
# PackedQMoETensor
# ---------------------------------------------------------------------------

class PackedQMoETensor:
    """Device-resident 2-bit packed matrix (qmoe-rs src/tensor.rs:16-121)."""

    def __init__(self, handle, ctx: Context, shape, scales):
        self._h = handle
        self.ctx = ctx
        self.shape = tuple(int(v) for v in shape)
        self.scales = scales

    @classmethod
    def from_bytes(cls, packed, shape: Tuple[int, int], scales,
                   ctx: Optional[Context] = None) -> "PackedQMoETensor":
        """PackedQMoETensor::from_bytes (src/tensor.rs:47-53)."""
        ctx = ctx or default_context()
        out_f, in_f = shape
        pp, kind, keep1 = _ptr(packed)
        sp, kind2, keep2 = _ptr(scales)
        if kind != kind2:
            raise ValueError("packed and scales must both be host or both device memory")
        if _is_cuda(packed):
            ctx.use_current_torch_stream()
        h = ctypes.c_void_p()
        capi.call("qmoe_packed_create", ctx.handle, pp, sp, int(out_f), int(in_f), kind,
                  ctypes.byref(h))
        return cls(h, ctx, shape, scales)

    def forward_simd(self, x):
        """PackedQMoETensor::forward_simd (src/tensor.rs:64-95): y[..., out]."""
        out_f, in_f = self.shape
        n = int(np.prod(x.shape)) if len(x.shape) else 0
        batch = n // in_f
        if batch * in_f != n:
            raise ValueError(
                f"Input tensor size {n} does not match batch_size * in_features = "
                f"{batch} * {in_f}")
        if _dtype_code(x) != capi.QMOE_DTYPE_F32:
            raise TypeError("forward_simd takes f32 activations (src/tensor.rs:72)")
        y = _empty_like_kind(x, tuple(x.shape[:-1]) + (out_f,), capi.QMOE_DTYPE_F32)
        xp, kind, keep = _ptr(x)
        yp, kind2, _ = _ptr(y)
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_packed_forward", self._h, xp, batch, yp, kind)
        return y

    def forward_simd_raw(self, x) -> np.ndarray:
        """forward_simd_raw (src/tensor.rs:99-121): flat f32 in, flat f32 out."""
        a = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        return self.forward_simd(a.reshape(-1, self.shape[1])).reshape(-1)

    def close(self):
        if getattr(self, "_h", None):
            capi.lib().qmoe_packed_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# MoE layer
# ---------------------------------------------------------------------------

@dataclass
class MoEConfig:
    """qmoe-rs MoEConfig (src/moe.rs:6-11) plus the routing extensions; the
    defaults of the extra fields give qmoe-rs's routing."""

    num_experts: int
    top_k: int
    hidden_dim: int
    intermediate_dim: int
    shared_intermediate_dim: int = 0
    scoring: int = capi.QMOE_SCORING_SOFTMAX
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0

    def to_c(self, has_bias: bool) -> capi.MoeConfigC:
        return capi.MoeConfigC(
            self.num_experts, self.top_k, self.hidden_dim, self.intermediate_dim,
            self.shared_intermediate_dim, self.scoring, self.n_group, self.topk_group,
            int(bool(self.norm_topk_prob)), float(self.routed_scaling_factor),
            int(bool(has_bias)), 0)


@dataclass
class PackedExpert:
    """(packed, scales) pairs of one expert (src/moe.rs:15-19)."""

    gate_proj: Tuple[object, object]
    up_proj: Tuple[object, object]
    down_proj: Tuple[object, object]

    @classmethod
    def from_triple(cls, t) -> "PackedExpert":
        return cls(tuple(t[0]), tuple(t[1]), tuple(t[2]))


def _expert_struct(ex: PackedExpert, keep: list) -> Tuple[capi.ExpertWeightsC, int]:
    vals = []
    kinds = set()
    for pk, sc in (ex.gate_proj, ex.up_proj, ex.down_proj):
        if not (torch is not None and isinstance(pk, torch.Tensor)):
            pk = np.ascontiguousarray(pk, dtype=np.uint8)
        if not (torch is not None and isinstance(sc, torch.Tensor)):
            sc = np.ascontiguousarray(sc, dtype=np.float32)
        p1, k1, a1 = _ptr(pk)
        p2, k2, a2 = _ptr(sc)
        keep += [a1, a2]
        kinds |= {k1, k2}
        vals += [p1, p2]
    if len(kinds) != 1:
        raise ValueError("all weights of a layer must be host or all device memory")
    return capi.ExpertWeightsC(*[v.value for v in vals]), kinds.pop()


class QMoELayer:
    """QMoELayer (src/moe.rs:23-130) with its optional SharedExpert, resident
    on one B200.  For expert parallelism pass expert_begin / the local slice
    of `experts`.  With no experts (qmoe-rs's empty `experts`, e.g. a
    flattened layer) the forward is the shared expert alone (zeros without
    one) and gate_weight may be None."""

    def __init__(self, config: MoEConfig, gate_weight, experts: Sequence[PackedExpert],
                 shared: Optional[PackedExpert] = None, bias=None,
                 expert_begin: int = 0, ctx: Optional[Context] = None):
        self.config = config
        self.ctx = ctx or default_context()
        self.expert_begin = int(expert_begin)
        self.expert_count = len(experts)
        keep: list = []
        kinds = set()
        gp = None
        if gate_weight is not None:
            if not (torch is not None and isinstance(gate_weight, torch.Tensor)):
                gate_weight = np.ascontiguousarray(gate_weight, dtype=np.float32)
            gp, gkind, ga = _ptr(gate_weight)
            keep.append(ga)
            kinds.add(gkind)
        elif len(experts):
            raise ValueError("a layer with routed experts needs its gate_weight")
        bp = None
        if bias is not None:
            if not (torch is not None and isinstance(bias, torch.Tensor)):
                bias = np.ascontiguousarray(bias, dtype=np.float32)
            bp, bkind, ba = _ptr(bias)
            keep.append(ba)
        arr = (capi.ExpertWeightsC * max(1, len(experts)))()
        for i, ex in enumerate(experts):
            if not isinstance(ex, PackedExpert):
                ex = PackedExpert.from_triple(ex)
            arr[i], k = _expert_struct(ex, keep)
            kinds.add(k)
        sh = None
        if shared is not None:
            if not isinstance(shared, PackedExpert):
                shared = PackedExpert.from_triple(shared)
            s, k = _expert_struct(shared, keep)
            kinds.add(k)
            sh = ctypes.pointer(s)
        if len(kinds) > 1:
            raise ValueError("all weights of a layer must be host or all device memory")
        kind = kinds.pop() if kinds else capi.QMOE_PTR_HOST
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        cfg = config.to_c(bias is not None)
        h = ctypes.c_void_p()
        capi.call("qmoe_layer_create", self.ctx.handle, ctypes.byref(cfg), gp, bp, arr,
                  self.expert_begin, self.expert_count, sh, kind, ctypes.byref(h))
        self._h = h
        del keep

    # -- qmoe-rs API ---------------------------------------------------------
    def forward(self, xs, return_routing: bool = False, out=None):
        """QMoELayer::forward + shared expert add (src/moe.rs:40-130,
        src/model.rs:386-389).  xs [T, H] f32 or bf16; `out` (optional) is a
        preallocated result of the same kind, dtype and shape."""
        T, H = xs.shape
        if H != self.config.hidden_dim:
            raise ValueError(f"hidden dim {H} != {self.config.hidden_dim}")
        dt = _dtype_code(xs)
        if out is None:
            out = _empty_like_kind(xs, (T, H), dt)
        K = self.config.top_k
        idx = w = None
        ip = wp = None
        if return_routing:
            idx = _empty_aux(xs, (T, K), np.int32, torch.int32 if torch else None)
            w = _empty_aux(xs, (T, K), np.float32, torch.float32 if torch else None)
            ip, wp = _ptr(idx)[0], _ptr(w)[0]
        xp, kind, keep = _ptr(xs)
        op, okind, _ = _ptr(out)
        if okind != kind:
            raise ValueError("x and out must both be host or both device memory")
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_forward", self._h, xp, dt, T, op, ip, wp, kind)
        if return_routing:
            return out, idx, w
        return out

    def route(self, xs):
        """Router only (src/moe.rs:51-82) -> (topk_idx [T,k] i32, topk_w [T,k] f32)."""
        T, _ = xs.shape
        K = self.config.top_k
        idx = _empty_aux(xs, (T, K), np.int32, torch.int32 if torch else None)
        w = _empty_aux(xs, (T, K), np.float32, torch.float32 if torch else None)
        xp, kind, keep = _ptr(xs)
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_route", self._h, xp, _dtype_code(xs), T, _ptr(idx)[0],
                  _ptr(w)[0], kind)
        return idx, w

    def forward_routed(self, xs, local_idx, weights):
        """Experts of this rank for rows with known routing (local ids, -1 = skip)."""
        R, H = xs.shape
        dt = _dtype_code(xs)
        out = _empty_like_kind(xs, (R, H), dt)
        xp, kind, k1 = _ptr(xs)
        ip, _, k2 = _ptr(local_idx)
        wp, _, k3 = _ptr(weights)
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_forward_routed", self._h, xp, dt, R, ip, wp, _ptr(out)[0], kind)
        return out

    def shared_forward(self, xs, out=None):
        """SharedExpert::forward (src/model.rs:325-347); with `out`, adds into it."""
        T, H = xs.shape
        dt = _dtype_code(xs)
        acc = out is not None
        if out is None:
            out = _empty_like_kind(xs, (T, H), dt)
        xp, kind, keep = _ptr(xs)
        op, _, _ = _ptr(out)
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_shared_forward", self._h, xp, dt, T, op, int(acc), kind)
        return out

    def set_norm(self, weight, bias, eps: float = 1e-6) -> None:
        """The decoder layer's post_attention_layernorm (src/model.rs:366-367):
        weight and bias [hidden_dim] f32."""
        keep = []
        ptrs = []
        kinds = set()
        for a in (weight, bias):
            if not (torch is not None and isinstance(a, torch.Tensor)):
                a = np.ascontiguousarray(a, dtype=np.float32)
            p, k, ka = _ptr(a)
            keep.append(ka)
            ptrs.append(p)
            kinds.add(k)
        if len(kinds) != 1:
            raise ValueError("weight and bias must both be host or both device memory")
        kind = kinds.pop()
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_set_norm", self._h, ptrs[0], ptrs[1], float(eps), kind)

    def forward_block(self, xs, return_routing: bool = False, out=None):
        """The MoE half of a decoder layer (src/model.rs:400-412): xs + moe(LN(xs))
        + shared(LN(xs)), with LN the post-attention LayerNorm set by set_norm."""
        T, H = xs.shape
        if H != self.config.hidden_dim:
            raise ValueError(f"hidden dim {H} != {self.config.hidden_dim}")
        dt = _dtype_code(xs)
        if out is None:
            out = _empty_like_kind(xs, (T, H), dt)
        K = self.config.top_k
        idx = w = None
        ip = wp = None
        if return_routing:
            idx = _empty_aux(xs, (T, K), np.int32, torch.int32 if torch else None)
            w = _empty_aux(xs, (T, K), np.float32, torch.float32 if torch else None)
            ip, wp = _ptr(idx)[0], _ptr(w)[0]
        xp, kind, keep = _ptr(xs)
        op, okind, _ = _ptr(out)
        if okind != kind:
            raise ValueError("x and out must both be host or both device memory")
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_layer_forward_block", self._h, xp, dt, T, op, ip, wp, kind)
        if return_routing:
            return out, idx, w
        return out

    def reserve(self, max_tokens: int) -> None:
        capi.call("qmoe_layer_reserve", self._h, int(max_tokens))

    def set_path(self, path: int) -> None:
        """Expert-product kernels: capi.QMOE_PATH_AUTO / _DECODE / _PREFILL / _DECODE_SPLIT."""
        capi.call("qmoe_layer_set_path", self._h, int(path))

    def set_profiling(self, enable: bool) -> None:
        capi.call("qmoe_layer_set_profiling", self._h, int(bool(enable)))

    def stage_times(self) -> dict:
        """Stage durations (ms) of the last forward run with profiling on."""
        buf = (ctypes.c_float * len(capi.STAGES))()
        n = ctypes.c_int()
        capi.call("qmoe_layer_stage_times", self._h, buf, len(capi.STAGES), ctypes.byref(n))
        return {capi.STAGES[i]: float(buf[i]) for i in range(n.value)}

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            capi.lib().qmoe_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BlockChain:
    """The layer loop of DeepSeekCoderV2::forward_next (src/model.rs:481-489)
    over the MoE halves of consecutive decoder layers (attention left out):
    x -> block_0 -> block_1 -> ..., each block a QMoELayer with its
    post-attention LayerNorm set.  Repeated calls with the same buffers replay
    one captured CUDA graph of all the layers' launches."""

    def __init__(self, layers: Sequence["QMoELayer"]):
        if not layers:
            raise ValueError("a chain needs at least one layer")
        self.layers = list(layers)
        self.ctx = self.layers[0].ctx
        arr = (ctypes.c_void_p * len(self.layers))(*[L.handle.value for L in self.layers])
        h = ctypes.c_void_p()
        capi.call("qmoe_chain_create", arr, len(self.layers), ctypes.byref(h))
        self._h = h

    def forward(self, xs, out=None):
        T, H = xs.shape
        dt = _dtype_code(xs)
        if out is None:
            out = _empty_like_kind(xs, (T, H), dt)
        xp, kind, keep = _ptr(xs)
        op, okind, _ = _ptr(out)
        if okind != kind:
            raise ValueError("x and out must both be host or both device memory")
        if kind == capi.QMOE_PTR_DEVICE:
            self.ctx.use_current_torch_stream()
        capi.call("qmoe_chain_forward", self._h, xp, dt, T, op, kind)
        return out

    def close(self):
        if getattr(self, "_h", None):
            capi.lib().qmoe_chain_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
