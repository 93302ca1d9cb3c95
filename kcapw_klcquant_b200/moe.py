"""Batched MoE layer on the device: router -> dispatch -> experts -> combine.

Thin host wrapper over the C ABI (``klc_moe_forward`` / ``klc_moe_experts``):
it owns a per-device workspace that grows on demand, builds the weight
descriptor once per layer, and passes raw pointers plus the current CUDA
stream.  All math runs in the CUDA kernels of libklcmoe.so.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass

import torch

from . import _lib
from .mxfp4_expert import PackedLayer

# One workspace per (device, stream): calls on different streams (or from
# different host threads on their own streams) never share scratch, while calls
# on one stream reuse it in stream order.
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}
# workspaces replaced by larger ones stay allocated: a CUDA graph captured
# while one was current still writes to it on replay
_RETIRED_WORKSPACES: list[torch.Tensor] = []
_WS_LOCK = threading.Lock()


def workspace(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """A device byte buffer of at least ``nbytes`` (256-byte aligned) for calls on
    ``stream`` (a raw ``cudaStream_t``; default: the device's current stream),
    reused by later calls on the same stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(idx).cuda_stream
    key = (idx, int(stream))
    with _WS_LOCK:
        ws = _WORKSPACES.get(key)
        if ws is None or ws.numel() < nbytes:
            if ws is not None:
                _RETIRED_WORKSPACES.append(ws)
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
            _WORKSPACES[key] = ws
    return ws


def as_bf16(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    if t.device == device and t.dtype == torch.bfloat16 and t.is_contiguous():
        return t
    return t.to(device=device, dtype=torch.bfloat16).contiguous()


@dataclass
class RouteBatch:
    """Routing of a token batch: expert ids int32 [T,k] (top-k order), bf16 weights [T,k]."""

    indices: torch.Tensor
    weights: torch.Tensor
    logits: torch.Tensor | None = None
    norms: torch.Tensor | None = None  # fp32 [T,k,2]: (||gated||, ||out||) per selected expert
    normed: torch.Tensor | None = None  # bf16 [T,H]: the next layer's input RMSNorm of the output (next_norm)
    next_indices: torch.Tensor | None = None  # int32 [T,k']: the next layer's routing of ``normed`` (next_router)
    next_weights: torch.Tensor | None = None  # bf16 [T,k']


class MoeLayer:
    """One MoE layer's device-resident weights plus the batched forward.

    ``packed`` holds the MXFP4 expert tensors; the dense tensors (router
    weight/bias, expert biases) are bf16 on the same device.
    """

    def __init__(
        self,
        packed: PackedLayer,
        router_weight: torch.Tensor,
        router_bias: torch.Tensor,
        gate_up_bias: torch.Tensor,
        down_bias: torch.Tensor,
        top_k: int = 4,
        swiglu_limit: float = 7.0,
        alpha: float = 1.702,
        path: str = "auto",
    ) -> None:
        dev = packed.gu_blocks.device
        self.device = dev
        self.packed = packed
        self.router_weight = as_bf16(router_weight, dev)
        self.router_bias = as_bf16(router_bias, dev)
        self.gate_up_bias = as_bf16(gate_up_bias, dev)
        self.down_bias = as_bf16(down_bias, dev)
        self.top_k = int(top_k)
        self.path = path
        self._last = threading.local()  # workspace + stream of this thread's last call
        E, H, I = packed.experts, packed.hidden, packed.intermediate
        if self.router_weight.shape != (E, H) or self.router_bias.shape != (E,):
            raise ValueError(f"router weight/bias must be [{E},{H}] / [{E}]")
        if self.gate_up_bias.shape != (E, 2 * I) or self.down_bias.shape != (E, H):
            raise ValueError(f"expert biases must be [{E},{2 * I}] / [{E},{H}]")
        self.weights = _lib.KlcWeights(
            packed.gu_blocks.data_ptr(), packed.gu_scales_t.data_ptr(), self.gate_up_bias.data_ptr(),
            packed.dn_blocks.data_ptr(), packed.dn_scales_t.data_ptr(), self.down_bias.data_ptr(),
            self.router_weight.data_ptr(), self.router_bias.data_ptr(), float(swiglu_limit), float(alpha),
            _lib.ptr(packed.gu_scales_mx), _lib.ptr(packed.dn_scales_mx),
            _lib.ptr(packed.gu_blocks_k128), _lib.ptr(packed.dn_blocks_k128),
            _lib.ptr(packed.gu_scales_t192), _lib.ptr(packed.dn_scales_t192),
        )

    @classmethod
    def from_tensors(cls, layer_idx: int, tensors: dict[str, torch.Tensor], device, top_k: int = 4, **kw) -> "MoeLayer":
        """Build from checkpoint-named tensors (``model.layers.{L}.mlp.*``)."""
        p = f"model.layers.{layer_idx}.mlp"
        dev = torch.device(device)
        packed = PackedLayer.from_checkpoint_tensors(
            tensors[f"{p}.experts.gate_up_proj_blocks"], tensors[f"{p}.experts.gate_up_proj_scales"],
            tensors[f"{p}.experts.down_proj_blocks"], tensors[f"{p}.experts.down_proj_scales"], dev,
        )
        return cls(packed, tensors[f"{p}.router.weight"], tensors[f"{p}.router.bias"], tensors[f"{p}.experts.gate_up_proj_bias"],
                   tensors[f"{p}.experts.down_proj_bias"], top_k=top_k, **kw)

    @property
    def experts(self) -> int:
        return self.packed.experts

    @property
    def hidden(self) -> int:
        return self.packed.hidden

    @property
    def intermediate(self) -> int:
        return self.packed.intermediate

    def dims(self, tokens: int, path: str | None = None) -> _lib.KlcDims:
        return _lib.KlcDims(int(tokens), self.hidden, self.intermediate, self.experts, self.top_k, _lib.PATH_CODE[path or self.path])

    def workspace_bytes(self, tokens: int, path: str | None = None) -> int:
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().klc_moe_workspace_size(ctypes.byref(self.dims(tokens, path)), ctypes.byref(n)))
        return int(n.value)

    def forward(
        self,
        x: torch.Tensor,
        precision: str = "bf16",
        adjust: torch.Tensor | None = None,
        return_logits: bool = False,
        return_norms: bool = False,
        residual: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        path: str | None = None,
        next_norm: tuple[torch.Tensor, float] | None = None,
        next_router: "MoeLayer | None" = None,
    ) -> tuple[torch.Tensor, RouteBatch]:
        """Router + experts + combine for ``x`` bf16 [T, H] -> (y bf16 [T, H], routing).

        ``next_norm=(weight, eps)`` also returns ``routing.normed`` =
        ``rms_norm(y, weight, eps)`` -- the executor's ``hidden += moe_out``
        followed by the next layer's input norm
        (streamed_transformer_executor.py:235,260) -- computed by the combine
        kernel itself.  ``next_router`` (the next layer, with ``next_norm``)
        routes ``normed`` for it as well (``routing.next_indices`` /
        ``next_weights``) in the same library call.
        """
        T = int(x.shape[0])
        x = as_bf16(x, self.device)
        dims = self.dims(T, path)
        k = self.top_k
        idx = torch.empty((T, k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, k), dtype=torch.bfloat16, device=self.device)
        logits = torch.empty((T, self.experts), dtype=torch.bfloat16, device=self.device) if return_logits else None
        norms = torch.empty((T, k, 2), dtype=torch.float32, device=self.device) if return_norms else None
        y = out if out is not None else torch.empty((T, self.hidden), dtype=torch.bfloat16, device=self.device)
        if residual is not None:
            residual = as_bf16(residual, self.device)
        if adjust is not None:
            adjust = adjust.to(device=self.device, dtype=torch.float32).contiguous()
        nbytes = self.workspace_bytes(T, path)
        stream = _lib.stream_ptr(self.device)
        ws = workspace(self.device, nbytes, stream)
        self._last.ws, self._last.stream = ws, stream
        normed = None
        with torch.cuda.device(self.device):
            if next_norm is None:
                _lib.check(
                    _lib.lib().klc_moe_forward(
                        ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), _lib.ptr(adjust),
                        _lib.PRECISION_CODE[precision], y.data_ptr(), idx.data_ptr(), w.data_ptr(), _lib.ptr(logits),
                        _lib.ptr(norms), _lib.ptr(residual), ws.data_ptr(), ws.numel(), stream,
                    )
                )
            else:
                norm_w = as_bf16(next_norm[0], self.device)
                if norm_w.numel() != self.hidden:
                    raise ValueError(f"next_norm weight must have {self.hidden} elements")
                normed = torch.empty_like(y)
                if next_router is None:
                    _lib.check(
                        _lib.lib().klc_moe_forward_rmsnorm(
                            ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), _lib.ptr(adjust),
                            _lib.PRECISION_CODE[precision], y.data_ptr(), idx.data_ptr(), w.data_ptr(), _lib.ptr(logits),
                            _lib.ptr(norms), _lib.ptr(residual), norm_w.data_ptr(), float(next_norm[1]), normed.data_ptr(),
                            ws.data_ptr(), ws.numel(), stream,
                        )
                    )
                else:
                    nr, nidx, nw = next_router.next_router_args(T)
                    _lib.check(
                        _lib.lib().klc_moe_forward_rmsnorm_route(
                            ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), _lib.ptr(adjust),
                            _lib.PRECISION_CODE[precision], y.data_ptr(), idx.data_ptr(), w.data_ptr(), _lib.ptr(logits),
                            _lib.ptr(norms), _lib.ptr(residual), norm_w.data_ptr(), float(next_norm[1]), normed.data_ptr(),
                            ctypes.byref(nr), ws.data_ptr(), ws.numel(), stream,
                        )
                    )
                    return y, RouteBatch(idx, w, logits, norms, normed, nidx, nw)
        if next_router is not None:
            raise ValueError("next_router needs next_norm")
        return y, RouteBatch(idx, w, logits, norms, normed)

    def next_router_args(self, T: int) -> tuple:
        """This layer's router as the previous layer's fused ``next_router``: (klc_next_router, idx, w)."""
        if self.router_weight.device != self.device:
            raise ValueError("router on another device")
        nidx = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device)
        nw = torch.empty((T, self.top_k), dtype=torch.bfloat16, device=self.device)
        nr = _lib.KlcNextRouter(self.router_weight.data_ptr(), self.router_bias.data_ptr(), self.experts, self.top_k,
                                nidx.data_ptr(), nw.data_ptr(), None)
        return nr, nidx, nw

    def experts_forward(
        self,
        x: torch.Tensor,
        indices: torch.Tensor,
        weights: torch.Tensor,
        precision: str = "bf16",
        return_norms: bool = False,
        residual: torch.Tensor | None = None,
        path: str | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Experts + combine for given routing (int32 [T,k], bf16 [T,k])."""
        T = int(x.shape[0])
        x = as_bf16(x, self.device)
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        w = weights.to(device=self.device, dtype=torch.bfloat16).contiguous()
        if idx.shape != (T, self.top_k) or w.shape != (T, self.top_k):
            raise ValueError(f"routing must be [{T},{self.top_k}]")
        dims = self.dims(T, path)
        norms = torch.empty((T, self.top_k, 2), dtype=torch.float32, device=self.device) if return_norms else None
        y = torch.empty((T, self.hidden), dtype=torch.bfloat16, device=self.device)
        if residual is not None:
            residual = as_bf16(residual, self.device)
        nbytes = self.workspace_bytes(T, path)
        stream = _lib.stream_ptr(self.device)
        ws = workspace(self.device, nbytes, stream)
        self._last.ws, self._last.stream = ws, stream
        with torch.cuda.device(self.device):
            _lib.check(
                _lib.lib().klc_moe_experts(
                    ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                    _lib.PRECISION_CODE[precision], y.data_ptr(), _lib.ptr(norms), _lib.ptr(residual),
                    ws.data_ptr(), ws.numel(), stream,
                )
            )
        return y, norms

    def experts_step(
        self,
        x: torch.Tensor,
        indices: torch.Tensor,
        weights: torch.Tensor,
        residual: torch.Tensor,
        next_norm: tuple[torch.Tensor, float],
        next_router: "MoeLayer | None" = None,
        precision: str = "bf16",
    ) -> tuple[torch.Tensor, RouteBatch]:
        """One stacked layer on routing computed by the previous layer: experts + combine +
        residual + the next layer's input RMSNorm (``routing.normed``) and, with
        ``next_router``, the next layer's routing of it (``routing.next_indices`` /
        ``next_weights``), all fused into the combine (klc_moe_experts_rmsnorm_route)."""
        T = int(x.shape[0])
        x = as_bf16(x, self.device)
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        w = weights.to(device=self.device, dtype=torch.bfloat16).contiguous()
        if idx.shape != (T, self.top_k) or w.shape != (T, self.top_k):
            raise ValueError(f"routing must be [{T},{self.top_k}]")
        residual = as_bf16(residual, self.device)
        norm_w = as_bf16(next_norm[0], self.device)
        dims = self.dims(T, None)
        y = torch.empty((T, self.hidden), dtype=torch.bfloat16, device=self.device)
        normed = torch.empty_like(y)
        nbytes = self.workspace_bytes(T, None)
        stream = _lib.stream_ptr(self.device)
        ws = workspace(self.device, nbytes, stream)
        self._last.ws, self._last.stream = ws, stream
        with torch.cuda.device(self.device):
            if next_router is None:
                _lib.check(_lib.lib().klc_moe_experts(
                    ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                    _lib.PRECISION_CODE[precision], y.data_ptr(), None, residual.data_ptr(), ws.data_ptr(), ws.numel(), stream))
                _lib.check(_lib.lib().klc_rms_norm(y.data_ptr(), norm_w.data_ptr(), T, self.hidden, float(next_norm[1]),
                                                   normed.data_ptr(), stream))
                return y, RouteBatch(idx, w, normed=normed)
            nr, nidx, nw = next_router.next_router_args(T)
            _lib.check(_lib.lib().klc_moe_experts_rmsnorm_route(
                ctypes.byref(dims), ctypes.byref(self.weights), x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                _lib.PRECISION_CODE[precision], y.data_ptr(), None, residual.data_ptr(), norm_w.data_ptr(), float(next_norm[1]),
                normed.data_ptr(), ctypes.byref(nr), ws.data_ptr(), ws.numel(), stream))
        return y, RouteBatch(idx, w, normed=normed, next_indices=nidx, next_weights=nw)

    def check_device_status(self) -> None:
        """Raise if a kernel of this thread's last call recorded a device-side fault.

        Reads the status word of the workspace that call used, on the stream it
        ran on (synchronises that stream)."""
        ws = getattr(self._last, "ws", None)
        if ws is None:
            return
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().klc_workspace_status(ws.data_ptr(), None, None, None, self._last.stream))


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Device RMSNorm with the reference's rounding (streamed_attention.py:27-28)."""
    x = x.contiguous()
    _lib.require_cuda(x)
    w = as_bf16(weight, x.device)
    if x.dtype != torch.bfloat16:
        raise ValueError("rms_norm expects bf16 activations")
    y = torch.empty_like(x)
    H = int(x.shape[-1])
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().klc_rms_norm(x.data_ptr(), w.data_ptr(), x.numel() // H, H, float(eps), y.data_ptr(), _lib.stream_ptr()))
    return y
