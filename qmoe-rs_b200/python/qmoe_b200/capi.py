"""ctypes binding of include/qmoe_b200.h.

Loads the in-tree lib/libqmoe_b200.so and raises if it is missing: there is
no fallback implementation behind this module.
"""
from __future__ import annotations

import ctypes
import os

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB_PATH = os.environ.get("QMOE_B200_LIB",
                          os.path.join(_PKG_ROOT, "lib", "libqmoe_b200.so"))
REPO_ROOT = os.path.dirname(_PKG_ROOT)
HEADER_PATH = os.path.join(REPO_ROOT, "include", "qmoe_b200.h")

QMOE_OK = 0
QMOE_ERR_INVALID = 1
QMOE_ERR_CUDA = 2
QMOE_ERR_UNSUPPORTED = 3
QMOE_ERR_NOMEM = 4
QMOE_PTR_DEVICE = 0
QMOE_PTR_HOST = 1
QMOE_DTYPE_F32 = 0
QMOE_DTYPE_BF16 = 1
QMOE_SCORING_SOFTMAX = 0
QMOE_SCORING_SIGMOID = 1
QMOE_PATH_AUTO = 0
QMOE_PATH_DECODE = 1
QMOE_PATH_PREFILL = 2
QMOE_PATH_DECODE_SPLIT = 3
QMOE_NOALLOC_MAX_BATCH = 16384
QMOE_NOALLOC_MAX_IN_FEATURES = 8192
QMOE_EP_HANDLE_BYTES = 64


class QmoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qmoe error {code}: {msg}")
        self.code = code


class MoeConfigC(ctypes.Structure):
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
        ("reserved", ctypes.c_int32),
    ]


class ExpertWeightsC(ctypes.Structure):
    _fields_ = [
        ("gate_packed", ctypes.c_void_p),
        ("gate_scales", ctypes.c_void_p),
        ("up_packed", ctypes.c_void_p),
        ("up_scales", ctypes.c_void_p),
        ("down_packed", ctypes.c_void_p),
        ("down_scales", ctypes.c_void_p),
    ]


# name -> (restype, argtypes); every function declared in the header
_P = ctypes.c_void_p
_I = ctypes.c_int
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_PP = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "qmoe_last_error": (ctypes.c_char_p, []),
    "qmoe_abi_version": (_I, []),
    "qmoe_ctx_create": (_I, [_I, _P, _PP]),
    "qmoe_ctx_destroy": (_I, [_P]),
    "qmoe_ctx_set_stream": (_I, [_P, _P]),
    "qmoe_ctx_synchronize": (_I, [_P]),
    "qmoe_packed_create": (_I, [_P, _P, _P, _I64, _I64, _I, _PP]),
    "qmoe_packed_destroy": (_I, [_P]),
    "qmoe_packed_shape": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "qmoe_packed_forward": (_I, [_P, _P, _I64, _P, _I]),
    "qmoe_quantize_pack": (_I, [_P, _P, _I64, _I64, _P, _I, _P, _I]),
    "qmoe_layer_create": (_I, [_P, ctypes.POINTER(MoeConfigC), _P, _P,
                               ctypes.POINTER(ExpertWeightsC), _I32, _I32,
                               ctypes.POINTER(ExpertWeightsC), _I, _PP]),
    "qmoe_layer_destroy": (_I, [_P]),
    "qmoe_layer_reserve": (_I, [_P, _I64]),
    "qmoe_layer_forward": (_I, [_P, _P, _I, _I64, _P, _P, _P, _I]),
    "qmoe_layer_route": (_I, [_P, _P, _I, _I64, _P, _P, _I]),
    "qmoe_layer_forward_routed": (_I, [_P, _P, _I, _I64, _P, _P, _P, _I]),
    "qmoe_layer_shared_forward": (_I, [_P, _P, _I, _I64, _P, _I, _I]),
    "qmoe_packed_forward_noalloc": (_I, [_I, _P, _P, _P, _I64, _I64, _P, _I64, _P]),
    "qmoe_layer_set_path": (_I, [_P, _I]),
    "qmoe_layer_set_norm": (_I, [_P, _P, _P, ctypes.c_float, _I]),
    "qmoe_layer_forward_block": (_I, [_P, _P, _I, _I64, _P, _P, _P, _I]),
    "qmoe_chain_create": (_I, [ctypes.POINTER(_P), _I, _PP]),
    "qmoe_chain_destroy": (_I, [_P]),
    "qmoe_chain_forward": (_I, [_P, _P, _I, _I64, _P, _I]),
    "qmoe_ep_plan": (_I, [_P, _P, _P, _I64, _I, _I, _I, _I64, _P, _P, _P, _P]),
    "qmoe_gather_rows": (_I, [_P, _P, _I, _I64, _P, _I64, _P]),
    "qmoe_combine_rows": (_I, [_P, _P, _I, _I64, _P, _I, _I64, _P, _P]),
    "qmoe_layer_forward_ep": (_I, [_P, _P, _I, _I64, _P, _I64, _P]),
    "qmoe_layer_route_plan": (_I, [_P, _P, _I, _I64, _P, _P, _I, _I, _I64, _P, _P, _P, _P]),
    "qmoe_layer_forward_ep_return": (_I, [_P, _P, _P, _I, _I64, _P, _I64, _P]),
    "qmoe_ep_finish": (_I, [_P, _P, _I64, _P, _P]),
    "qmoe_ep_peer_create": (_I, [_P, _I, _I, _I64, _I64, _I, _I, _PP]),
    "qmoe_ep_peer_destroy": (_I, [_P]),
    "qmoe_ep_peer_handle": (_I, [_P, _P]),
    "qmoe_ep_peer_connect": (_I, [_P, _P]),
    "qmoe_ep_peer_buffers": (_I, [_P, _PP, _PP, _PP]),
    "qmoe_ep_dispatch": (_I, [_P, _P, _I64, _P, _P, _P]),
    "qmoe_ep_wait": (_I, [_P, _I]),
    "qmoe_ep_return": (_I, [_P, _P]),
    "qmoe_layer_set_profiling": (_I, [_P, _I]),
    "qmoe_layer_stage_times": (_I, [_P, ctypes.POINTER(ctypes.c_float), _I,
                                    ctypes.POINTER(ctypes.c_int)]),
}

STAGES = ("router", "permute", "quant_up", "gate_up", "quant_down", "down", "combine")

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if the CUDA build is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} not found: build it with `python qmoe-rs_b200/build.py` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != QMOE_OK:
        msg = lib().qmoe_last_error()
        raise QmoeError(rc, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
