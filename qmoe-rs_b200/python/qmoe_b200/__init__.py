"""qmoe_b200: B200-native (sm_100a) 2-bit MoE layer for qmoe-rs.

The compute lives in lib/libqmoe_b200.so (hand-written CUDA for sm_100a,
C ABI in include/qmoe_b200.h); this package is the host-side binding.
"""
from . import capi
from .capi import QmoeError
from .layer import (BlockChain, Context, MoEConfig, PackedExpert, PackedQMoETensor, QMoELayer,
                    default_context)
from . import quantize
from .ep import ExpertParallelMoE, TorchComm

__all__ = ["capi", "QmoeError", "BlockChain", "Context", "MoEConfig", "PackedExpert",
           "PackedQMoETensor", "QMoELayer", "default_context", "quantize",
           "ExpertParallelMoE", "TorchComm"]
