"""ctypes binding of libklcmoe.so (the C ABI declared in include/klc_moe.h).

The library is built in-tree by ``kcapw_klcquant_b200.build``.  Loading fails
loudly when it is missing: there is no CPU fallback for any MoE math.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libklcmoe.so"

KLC_OK = 0
KLC_ERR_INVALID = 1
KLC_ERR_UNSUPPORTED = 2
KLC_ERR_WORKSPACE = 3
KLC_ERR_CUDA = 4
KLC_ERR_DEVICE_TIMEOUT = 5
KLC_ERR_DEVICE_FAULT = 6
KLC_ERR_NCCL = 7

KLC_BF16, KLC_F16, KLC_F32 = 0, 1, 2
KLC_PREC_FP32, KLC_PREC_BF16 = 0, 1
KLC_PATH_AUTO, KLC_PATH_SIMT, KLC_PATH_TC = 0, 1, 2

DTYPE_CODE = {torch.bfloat16: KLC_BF16, torch.float16: KLC_F16, torch.float32: KLC_F32}
PRECISION_CODE = {"fp32": KLC_PREC_FP32, "bf16": KLC_PREC_BF16}
PATH_CODE = {"auto": KLC_PATH_AUTO, "simt": KLC_PATH_SIMT, "tc": KLC_PATH_TC}


class KlcError(RuntimeError):
    """A libklcmoe call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[klc status {status}] {message}")
        self.status = status


class KlcDims(ctypes.Structure):
    _fields_ = [
        ("tokens", c_int64),
        ("hidden", c_int64),
        ("intermediate", c_int64),
        ("experts", c_int64),
        ("top_k", c_int32),
        ("path", c_int32),
    ]


class KlcLocalityConfig(ctypes.Structure):
    """klc_locality_config: RoutingLocalityConfig's fields plus the router's experts_per_token."""

    _fields_ = [
        ("sticky_strength", ctypes.c_double),
        ("sticky_candidate_margin", ctypes.c_double),
        ("max_sticky_bonus", ctypes.c_double),
        ("exploration_margin", ctypes.c_double),
        ("cache_aware_strength", ctypes.c_double),
        ("sticky_decay", ctypes.c_double),
        ("workload_window", ctypes.c_double),
        ("semantic_guard", c_int32),
        ("min_raw_overlap", c_int32),
        ("max_hot_experts", c_int32),
        ("prediction_window", c_int32),
        ("predictive_prefetch", c_int32),
        ("experts_per_token", c_int32),
    ]


class KlcNextRouter(ctypes.Structure):
    """klc_next_router: the next layer's router, run on the normalised rows by the combine."""

    _fields_ = [
        ("router_w", c_void_p),
        ("router_b", c_void_p),
        ("experts", c_int64),
        ("k", c_int),
        ("out_idx", c_void_p),
        ("out_w", c_void_p),
        ("out_logits", c_void_p),
    ]


class KlcWeights(ctypes.Structure):
    _fields_ = [
        ("gu_blocks", c_void_p),
        ("gu_scales_t", c_void_p),
        ("gu_bias", c_void_p),
        ("dn_blocks", c_void_p),
        ("dn_scales_t", c_void_p),
        ("dn_bias", c_void_p),
        ("router_w", c_void_p),
        ("router_b", c_void_p),
        ("swiglu_limit", c_float),
        ("alpha", c_float),
        ("gu_scales_mx", c_void_p),
        ("dn_scales_mx", c_void_p),
        ("gu_blocks_k128", c_void_p),
        ("dn_blocks_k128", c_void_p),
        ("gu_scales_t192", c_void_p),
        ("dn_scales_t192", c_void_p),
    ]


# name -> argtypes (every entry point returns int, except klc_last_error)
SIGNATURES: dict[str, list] = {
    "klc_version": [],
    "klc_device_sm_count": [POINTER(c_int)],
    "klc_launch_count": [POINTER(ctypes.c_uint64)],
    "klc_struct_sizes": [POINTER(c_size_t), POINTER(c_size_t)],
    "klc_struct_size": [c_int, POINTER(c_size_t)],
    "klc_set_pdl": [c_int],
    "klc_set_pair_tiles": [c_int],
    "klc_set_fused_quantize": [c_int],
    "klc_selftest_wait_timeout": [c_int64, POINTER(c_int), POINTER(c_int), c_void_p],
    "klc_capabilities": [POINTER(c_int)],
    "klc_mxfp4_dequant": [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p],
    "klc_mxfp4_transpose_scales": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "klc_mxfp4_scales_mx_bytes": [c_int64, c_int64, c_int64, POINTER(c_size_t)],
    "klc_mxfp4_pad_k128": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "klc_mxfp4_scales_tile_bytes": [c_int64, c_int64, c_int64, c_int, POINTER(c_size_t)],
    "klc_mxfp4_scales_tile": [c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p],
    "klc_mxfp4_scales_mx": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "klc_mx_quantize_rows": [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "klc_router_status": [POINTER(c_int), POINTER(c_int), c_void_p],
    "klc_router_topk": [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "klc_select_softmax": [c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p],
    "klc_locality_state_bytes": [c_int64, c_int, POINTER(c_size_t)],
    "klc_locality_route": [POINTER(KlcLocalityConfig), c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p, c_size_t,
                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "klc_moe_workspace_size": [POINTER(KlcDims), POINTER(c_size_t)],
    "klc_moe_experts": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_moe_experts_noalloc": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "klc_moe_noalloc_scratch_bytes": [POINTER(c_size_t)],
    "klc_moe_noalloc_status": [POINTER(c_int), POINTER(c_int), POINTER(c_int), c_void_p],
    "klc_moe_forward": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_moe_combine": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p, c_void_p],
    "klc_moe_combine_rmsnorm": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p],
    "klc_moe_forward_rmsnorm": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_moe_forward_rmsnorm_route": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, POINTER(KlcNextRouter), c_void_p,
                                      c_size_t, c_void_p],
    "klc_moe_experts_rmsnorm_route": [POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_float, c_void_p, POINTER(KlcNextRouter), c_void_p, c_size_t, c_void_p],
    "klc_moe_combine_rmsnorm_route": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p, c_float, c_void_p,
                                      c_void_p, POINTER(KlcNextRouter), c_void_p],
    "klc_moe_bias_only": [c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "klc_moe_permute": [c_void_p, c_int64, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_size_t, c_void_p],
    "klc_ep_pack": [c_void_p, c_int64, c_int, c_int64, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_workspace_status": [c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int), c_void_p],
    "klc_stage_timing": [c_int],
    "klc_stage_times": [POINTER(c_float), c_int, POINTER(c_int)],
    "klc_ep_create": [c_int, c_int, c_int64, c_int, c_int64, c_int64, POINTER(c_void_p)],
    "klc_ep_arena_bytes": [c_void_p, POINTER(c_size_t)],
    "klc_ep_ipc_handle": [c_void_p, c_void_p],
    "klc_ep_connect": [c_void_p, c_void_p],
    "klc_ep_set_wait_limit_ns": [c_void_p, ctypes.c_uint64],
    "klc_ep_set_fused_return": [c_void_p, c_int],
    "klc_ep_workspace_size": [c_void_p, POINTER(KlcDims), POINTER(c_size_t)],
    "klc_ep_dispatch": [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_ep_experts": [c_void_p, POINTER(KlcDims), POINTER(KlcWeights), c_int, c_void_p, c_size_t, c_void_p],
    "klc_ep_combine": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p],
    "klc_ep_combine_route": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                             POINTER(KlcNextRouter), c_void_p],
    "klc_ep_forward": [c_void_p, POINTER(KlcDims), POINTER(KlcWeights), c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                       c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "klc_ep_status": [c_void_p, c_void_p, POINTER(c_int), POINTER(c_int), c_void_p],
    "klc_ep_received_rows": [c_void_p, POINTER(c_int64), c_void_p],
    "klc_ep_destroy": [c_void_p],
    "klc_rms_norm": [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p],
    "klc_runtime_dequant": [c_int, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p, c_int, c_void_p],
}

_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libklcmoe.so once and declare its signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m kcapw_klcquant_b200.build` "
            "(or __graft_entry__.build()); the MoE path has no CPU fallback"
        )
    # torch loads the CUDA runtime and initialises the driver first
    torch.cuda.is_available()
    h = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_GLOBAL if hasattr(os, "RTLD_GLOBAL") else 0)
    for name, args in SIGNATURES.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = c_int
    h.klc_last_error.argtypes = []
    h.klc_last_error.restype = c_char_p
    # the structures passed by pointer must have the library's layout
    for which, struct in enumerate((KlcDims, KlcWeights, KlcLocalityConfig, KlcNextRouter)):
        n = c_size_t(0)
        if h.klc_struct_size(which, ctypes.byref(n)) != KLC_OK or n.value != ctypes.sizeof(struct):
            raise ImportError(f"{LIB_PATH} was built with another {struct.__name__} layout ({n.value} B) than this "
                              f"binding ({ctypes.sizeof(struct)} B): rebuild it")
    _LIB = h
    return h


def capabilities() -> set[str]:
    """Expert paths compiled into the library ({"simt", "tc"})."""
    f = c_int(0)
    check(lib().klc_capabilities(ctypes.byref(f)))
    return {name for bit, name in ((1, "simt"), (2, "tc")) if f.value & bit}


def check(status: int) -> None:
    if status == KLC_OK:
        return
    msg = (lib().klc_last_error() or b"").decode(errors="replace")
    if status == KLC_ERR_INVALID:
        raise ValueError(msg)
    raise KlcError(status, msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("kcapw_klcquant_b200 runs on CUDA devices only (no CPU fallback); got a CPU tensor")
        if t is not None and not t.is_contiguous():
            raise ValueError("kcapw_klcquant_b200 expects contiguous tensors")


def launch_count() -> int:
    """Kernels libklcmoe.so has launched in this process so far."""
    n = ctypes.c_uint64(0)
    check(lib().klc_launch_count(ctypes.byref(n)))
    return int(n.value)


STAGES = ("router", "permute", "gate_up", "down", "combine")


def stage_timing(enable: bool) -> None:
    check(lib().klc_stage_timing(1 if enable else 0))


def stage_times() -> dict[str, float]:
    """Milliseconds per stage of the last layer call on this thread (needs stage_timing(True))."""
    buf = (c_float * len(STAGES))()
    n = c_int(0)
    check(lib().klc_stage_times(buf, len(STAGES), ctypes.byref(n)))
    return {name: float(buf[i]) for i, name in enumerate(STAGES) if buf[i] >= 0}
