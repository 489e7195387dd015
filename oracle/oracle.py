"""ctypes front end of the CPU oracle (qmoe_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / --impl reference legs, always as the checker (or the
timed CPU restatement), never by the qmoe_b200 package.

Each wrapper names the qmoe-rs function it restates (paths relative to the
qmoe-rs project root):
  dequant_dot      src/simd.rs:6-45
  packed_forward   src/tensor.rs:64-95
  gate_logits      pinned order standing in for candle's matmul, src/moe.rs:51
  route            src/moe.rs:57-82 (+ DeepSeek-V2/V3 routing extensions)
  moe_forward      src/moe.rs:40-130
  shared_forward   src/model.rs:325-347
  layer_forward    src/model.rs:386-389 (moe_out + shared_out)
  layernorm        post_attention_layernorm, src/model.rs:366-367, :401-403
                   (pinned order standing in for candle's layer_norm)
  block_forward    the MoE half of DecoderLayer::forward_*, src/model.rs:400-412
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libqmoe_oracle.so")

REDUCE_ORDERED = 0
REDUCE_PAIRWISE = 1
SCORING_SOFTMAX = 0
SCORING_SIGMOID = 1


class QoConfig(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("hidden_dim", ctypes.c_int32),
        ("intermediate_dim", ctypes.c_int32),
        ("shared_intermediate_dim", ctypes.c_int32),
        ("scoring", ctypes.c_int32),
        ("n_group", ctypes.c_int32),
        ("topk_group", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
        ("has_bias", ctypes.c_int32),
        ("reduce_mode", ctypes.c_int32),
    ]


@dataclass
class MoEConfig:
    """Mirror of qmoe-rs MoEConfig (src/moe.rs:6-11) plus routing extensions."""

    num_experts: int
    top_k: int
    hidden_dim: int
    intermediate_dim: int
    shared_intermediate_dim: int = 0
    scoring: int = SCORING_SOFTMAX
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0
    reduce_mode: int = REDUCE_ORDERED

    def c(self, has_bias: bool) -> QoConfig:
        return QoConfig(
            self.num_experts, self.top_k, self.hidden_dim, self.intermediate_dim,
            self.shared_intermediate_dim, self.scoring, self.n_group,
            self.topk_group, int(self.norm_topk_prob),
            float(self.routed_scaling_factor), int(has_bias), self.reduce_mode)


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, no reference sources)."""
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH)
            < os.path.getmtime(os.path.join(_HERE, "qmoe_oracle.c"))):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "all"],
                       check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.qo_dequant_dot.restype = ctypes.c_float
        L.qo_dequant_dot.argtypes = [P, i64, P, i64, ctypes.c_float, ctypes.c_int]
        L.qo_packed_forward.restype = None
        L.qo_packed_forward.argtypes = [P, P, i64, i64, P, i64, P, ctypes.c_int]
        L.qo_gate_logits.restype = None
        L.qo_gate_logits.argtypes = [P, P, i64, i64, i64, P]
        L.qo_exp.restype = ctypes.c_float
        L.qo_exp.argtypes = [ctypes.c_float]
        L.qo_sigmoid.restype = ctypes.c_float
        L.qo_sigmoid.argtypes = [ctypes.c_float]
        L.qo_route.restype = ctypes.c_int
        L.qo_route.argtypes = [ctypes.POINTER(QoConfig), P, P, i64, P, P]
        L.qo_moe_forward.restype = ctypes.c_int
        L.qo_moe_forward.argtypes = [ctypes.POINTER(QoConfig), P, P, P, P, P, i64,
                                     P, P, P, ctypes.c_int]
        L.qo_layer_forward.restype = ctypes.c_int
        L.qo_layer_forward.argtypes = [ctypes.POINTER(QoConfig), P, P, P, P, P, P,
                                       P, i64, P, P, P, ctypes.c_int]
        L.qo_shared_forward.restype = None
        L.qo_shared_forward.argtypes = [P, P, P, P, P, P, i64, i64, P, i64, P,
                                        ctypes.c_int, ctypes.c_int]
        L.qo_experts_forward.restype = None
        L.qo_experts_forward.argtypes = [ctypes.POINTER(QoConfig), P, P, P, i64, P, P, P,
                                         ctypes.c_int]
        L.qo_layernorm.restype = None
        L.qo_layernorm.argtypes = [P, P, P, ctypes.c_float, i64, i64, ctypes.c_int, P]
        L.qo_dequantize.restype = None
        L.qo_dequantize.argtypes = [P, P, i64, i64, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


def dequant_dot(packed, act, scale: float, reduce_mode: int = REDUCE_ORDERED) -> float:
    packed, act = _u8(packed), _f32(act)
    return float(lib().qo_dequant_dot(_p(packed), packed.size, _p(act), act.size,
                                      ctypes.c_float(scale), reduce_mode))


def packed_forward(packed, scales, shape, x, reduce_mode: int = REDUCE_ORDERED):
    """Y[..., out] for X[..., in] (forward_simd, src/tensor.rs:64-95)."""
    out_f, in_f = shape
    packed, scales = _u8(packed), _f32(scales)
    x = _f32(x)
    batch = x.size // in_f
    if batch * in_f != x.size:
        raise ValueError("input size does not match batch * in_features")
    y = np.empty(x.shape[:-1] + (out_f,), np.float32)
    lib().qo_packed_forward(_p(packed), _p(scales), out_f, in_f, _p(x), batch,
                            _p(y), reduce_mode)
    return y


def gate_logits(x, gate_w):
    x, gate_w = _f32(x), _f32(gate_w)
    T, H = x.shape
    E = gate_w.shape[0]
    out = np.empty((T, E), np.float32)
    lib().qo_gate_logits(_p(x), _p(gate_w), T, E, H, _p(out))
    return out


def qexp(v: float) -> float:
    return float(lib().qo_exp(ctypes.c_float(v)))


def sigmoid(v: float) -> float:
    return float(lib().qo_sigmoid(ctypes.c_float(v)))


def route(cfg: MoEConfig, logits, bias=None):
    logits = _f32(logits)
    T = logits.shape[0]
    idx = np.empty((T, cfg.top_k), np.int32)
    w = np.empty((T, cfg.top_k), np.float32)
    b = _f32(bias) if bias is not None else None
    c = cfg.c(b is not None)
    rc = lib().qo_route(ctypes.byref(c), _p(logits), _p(b) if b is not None else None,
                        T, _p(idx), _p(w))
    if rc != 0:
        raise ValueError("invalid routing configuration")
    return idx, w


def _weight_tables(experts):
    """experts: list of ((packed, scales) gate, up, down) -> pointer tables."""
    keep = []
    packed_ptrs = (ctypes.c_void_p * (3 * len(experts)))()
    scale_ptrs = (ctypes.c_void_p * (3 * len(experts)))()
    for e, ex in enumerate(experts):
        for j, (pk, sc) in enumerate(ex):
            pk, sc = _u8(pk), _f32(sc)
            keep += [pk, sc]
            packed_ptrs[3 * e + j] = pk.ctypes.data
            scale_ptrs[3 * e + j] = sc.ctypes.data
    return packed_ptrs, scale_ptrs, keep


def layer_forward(cfg: MoEConfig, gate_w, experts, x, shared=None, bias=None,
                  nthreads: int = 1):
    """Routed experts (src/moe.rs:40-130) plus optional shared expert
    (src/model.rs:325-347) added as in src/model.rs:386-389.

    experts: list of E entries ((gate_packed, gate_scales), (up_p, up_s),
    (down_p, down_s)); shared: the same triple or None.
    Returns (out [T,H] f32, topk_idx [T,k] i32, topk_w [T,k] f32)."""
    x = _f32(x)
    gate_w = _f32(gate_w)
    T = x.shape[0]
    out = np.empty((T, cfg.hidden_dim), np.float32)
    idx = np.empty((T, cfg.top_k), np.int32)
    w = np.empty((T, cfg.top_k), np.float32)
    pp, sp, keep = _weight_tables(experts)
    b = _f32(bias) if bias is not None else None
    c = cfg.c(b is not None)
    if shared is not None:
        spp, ssp, keep2 = _weight_tables([shared])
        keep += keep2
    else:
        spp = ssp = None
    rc = lib().qo_layer_forward(ctypes.byref(c), _p(gate_w),
                                _p(b) if b is not None else None, pp, sp, spp, ssp,
                                _p(x), T, _p(out), _p(idx), _p(w), nthreads)
    if rc != 0:
        raise ValueError("invalid routing configuration")
    del keep
    return out, idx, w


def moe_forward(cfg: MoEConfig, gate_w, experts, x, bias=None, nthreads: int = 1):
    """Routed experts only (QMoELayer::forward, src/moe.rs:40-130)."""
    x = _f32(x)
    gate_w = _f32(gate_w)
    T = x.shape[0]
    out = np.empty((T, cfg.hidden_dim), np.float32)
    idx = np.empty((T, cfg.top_k), np.int32)
    w = np.empty((T, cfg.top_k), np.float32)
    pp, sp, keep = _weight_tables(experts)
    b = _f32(bias) if bias is not None else None
    c = cfg.c(b is not None)
    rc = lib().qo_moe_forward(ctypes.byref(c), _p(gate_w),
                              _p(b) if b is not None else None, pp, sp, _p(x), T,
                              _p(out), _p(idx), _p(w), nthreads)
    if rc != 0:
        raise ValueError("invalid routing configuration")
    del keep
    return out, idx, w


def experts_forward(cfg: MoEConfig, experts, x, idx, w, nthreads: int = 1):
    """Routed experts for given routing (expert half of src/moe.rs:84-129);
    idx [R, k] expert ids or -1, w [R, k]."""
    x = _f32(x)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    w = _f32(w)
    R = x.shape[0]
    out = np.empty((R, cfg.hidden_dim), np.float32)
    pp, sp, keep = _weight_tables(experts)
    c = cfg.c(False)
    lib().qo_experts_forward(ctypes.byref(c), pp, sp, _p(x), R, _p(idx), _p(w), _p(out),
                             nthreads)
    del keep
    return out


def shared_forward(shared, x, hidden_dim: int, shared_dim: int,
                   reduce_mode: int = REDUCE_ORDERED, nthreads: int = 1):
    x = _f32(x)
    T = x.shape[0]
    (gp, gs), (up, us), (dp, ds) = [(_u8(a), _f32(b)) for a, b in shared]
    out = np.empty((T, hidden_dim), np.float32)
    lib().qo_shared_forward(_p(gp), _p(gs), _p(up), _p(us), _p(dp), _p(ds),
                            hidden_dim, shared_dim, _p(x), T, _p(out), reduce_mode,
                            nthreads)
    return out


def dequantize(packed, scales, shape):
    out_f, in_f = shape
    packed, scales = _u8(packed), _f32(scales)
    w = np.empty((out_f, in_f), np.float32)
    lib().qo_dequantize(_p(packed), _p(scales), out_f, in_f, _p(w))
    return w


def layernorm(x, w, b, eps: float = 1e-6, round_bf16: bool = False):
    """Pinned-order LayerNorm of the rows of x (see qo_layernorm)."""
    x = _f32(x)
    w, b = _f32(w), _f32(b)
    T, H = x.shape
    y = np.empty_like(x)
    lib().qo_layernorm(_p(x), _p(w), _p(b), ctypes.c_float(eps), T, H, int(round_bf16), _p(y))
    return y


def block_forward(cfg: MoEConfig, gate_w, experts, x, ln_w, ln_b, eps: float = 1e-6, shared=None,
                  bias=None, nthreads: int = 1, round_bf16: bool = False):
    """The MoE half of a decoder layer (src/model.rs:400-412): y =
    post_attention_layernorm(x); out = x + (moe(y) + shared(y)).  With
    round_bf16 the normalised rows are rounded to bf16 first (a bf16
    forward's router and experts read them so).  Returns (out, idx, w)."""
    x = _f32(x)
    y = layernorm(x, ln_w, ln_b, eps, round_bf16)
    moe, idx, w = layer_forward(cfg, gate_w, experts, y, shared=shared, bias=bias, nthreads=nthreads)
    return (x + moe).astype(np.float32), idx, w
