"""B200-native MoE block for KLCquant: router, dispatch, MXFP4 SwiGLU experts, combine.

Drop-in modules mirror the reference's (klcquant) module names:
``streamed_moe_router``, ``mxfp4_expert``, ``runtime_dequantizer``.  All MoE
math runs in the CUDA kernels of ``libklcmoe.so`` (C ABI in include/klc_moe.h).
"""
from .mxfp4_expert import FP4_VALUES, ExpertCacheStats, Mxfp4ExpertStore, PackedLayer, dequantize_mxfp4_matrix
from .moe import MoeLayer, RouteBatch, rms_norm
from .runtime_dequantizer import QuantizedTensorMeta, RuntimeDequantizer, parse_bool
from .streamed_moe_router import RouterStats, RoutingLocalityConfig, StreamedMoERouter

__all__ = [
    "FP4_VALUES",
    "ExpertCacheStats",
    "Mxfp4ExpertStore",
    "PackedLayer",
    "dequantize_mxfp4_matrix",
    "MoeLayer",
    "RouteBatch",
    "rms_norm",
    "QuantizedTensorMeta",
    "RuntimeDequantizer",
    "parse_bool",
    "RouterStats",
    "RoutingLocalityConfig",
    "StreamedMoERouter",
]
