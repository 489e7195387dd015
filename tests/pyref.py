"""A second, independent restatement of qmoe-rs's MoE path in plain Python.

Scalar float32 arithmetic through numpy scalars and glibc's expf / fmaf
(called with ctypes, the same libm Rust's f32 methods use on Linux).  It is
slow and only runs on tiny shapes; its job is to cross-check the C oracle
(oracle/qmoe_oracle.c) bit for bit.  Citations are qmoe-rs paths.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import functools

import numpy as np

f32 = np.float32
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_libm.fmaf.restype = ctypes.c_float
_libm.fmaf.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]


def expf(v) -> np.float32:
    return f32(_libm.expf(float(v)))


def fmaf(a, b, c) -> np.float32:
    return f32(_libm.fmaf(float(a), float(b), float(c)))


def dequant_dot(packed, act, scale, pairwise=False):
    """src/simd.rs:6-45, lane by lane."""
    lanes = [f32(0.0)] * 4
    nb = min(len(packed), len(act) // 4)
    for i in range(nb):
        b = int(packed[i])
        for j in range(4):
            w = f32(f32((b >> (2 * j)) & 3) - f32(1.0))
            lanes[j] = f32(lanes[j] + f32(w * f32(act[4 * i + j])))
    if pairwise:
        s = f32(f32(lanes[0] + lanes[1]) + f32(lanes[2] + lanes[3]))
    else:
        s = f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
    return f32(s * f32(scale))


def packed_forward(packed, scales, shape, x):
    """src/tensor.rs:64-95 for x [B, in]."""
    out_f, in_f = shape
    bpr = in_f // 4
    y = np.zeros((x.shape[0], out_f), np.float32)
    for b in range(x.shape[0]):
        for o in range(out_f):
            y[b, o] = dequant_dot(packed[o * bpr:(o + 1) * bpr], x[b], scales[o])
    return y


def gate_logits(x, gw, chunk=64):
    """The pinned logit order (chunked fmaf chains, summed chunk by chunk)."""
    T, H = x.shape
    E = gw.shape[0]
    out = np.zeros((T, E), np.float32)
    for t in range(T):
        for e in range(E):
            total = f32(0.0)
            for c0 in range(0, H, chunk):
                acc = f32(0.0)
                for k in range(c0, min(H, c0 + chunk)):
                    acc = fmaf(x[t, k], gw[e, k], acc)
                total = f32(total + acc)
            out[t, e] = total
    return out


def route_softmax(logits, top_k):
    """src/moe.rs:60-81: stable sort descending, softmax over all E summed in
    sorted order, first top_k, no renormalisation."""
    T, E = logits.shape
    idx = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), np.float32)
    for t in range(T):
        row = [(e, f32(logits[t, e])) for e in range(E)]
        row.sort(key=functools.cmp_to_key(
            lambda a, b: -1 if a[1] > b[1] else (1 if a[1] < b[1] else 0)))
        mx = f32(-np.inf)
        for _, v in row:
            mx = max(mx, v)
        s = f32(0.0)
        for _, v in row:
            s = f32(s + expf(f32(v - mx)))
        for j in range(top_k):
            e, v = row[j]
            idx[t, j] = e
            w[t, j] = f32(expf(f32(v - mx)) / s)
    return idx, w


def swiglu(g, u):
    """src/moe.rs:109-115."""
    swish = f32(g * f32(f32(1.0) / f32(f32(1.0) + expf(-g))))
    return f32(swish * u)


def moe_forward(E, top_k, H, I, gate_w, experts, x):
    """src/moe.rs:40-130 with the reference's expert-outer loop."""
    T = x.shape[0]
    logits = gate_logits(x, gate_w)
    idx, wts = route_softmax(logits, top_k)
    bins = [[] for _ in range(E)]
    for t in range(T):
        for j in range(top_k):
            bins[idx[t, j]].append((t, wts[t, j]))
    out = np.zeros((T, H), np.float32)
    for e in range(E):
        (gp, gs), (up, us), (dp, ds) = experts[e]
        for t, w in bins[e]:
            g = packed_forward(gp, gs, (I, H), x[t:t + 1])[0]
            u = packed_forward(up, us, (I, H), x[t:t + 1])[0]
            act = np.array([swiglu(g[i], u[i]) for i in range(I)], np.float32)
            d = packed_forward(dp, ds, (H, I), act[None])[0]
            for h in range(H):
                out[t, h] = f32(out[t, h] + f32(d[h] * w))
    return out, idx, wts
