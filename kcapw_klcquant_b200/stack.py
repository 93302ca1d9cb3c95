"""A stack of MoE blocks with the executor's RMSNorm and residual add between them.

The reference runs each transformer layer as attention, then
``post = rms_norm(hidden, ...)``, ``moe_out = router.route(..., post, ...)``
and ``hidden += moe_out`` (streamed_transformer_executor.py:231-275, rms_norm
at streamed_attention.py:27-28).  :class:`MoeStack` is the MoE half of that
layer loop over many layers and a whole batch of tokens at once:

    normed = rms_norm(hidden, norm[0])
    for every layer L:
        hidden = hidden + moe_L(normed)             # the combine adds the residual
        normed = rms_norm(hidden, norm[L + 1])      # ... and normalises for layer L+1

with the residual add and the next layer's norm fused into each layer's
combine kernel, so a layer is one MoE call.  With ``fuse_router`` the next
layer's router also runs in that call (the same kernels; a layer after the
first is then one experts-and-combine call on routing its predecessor already
computed).  Layers are :class:`MoeLayer` (one GPU) or
:class:`ExpertParallelMoe` with the peer-memory exchange (experts sharded over
the GPUs of a node); both are free of host synchronisation, so
:meth:`MoeStack.capture` records a whole decode step of all layers as one CUDA
graph and :meth:`MoeStack.replay` runs it.
"""
from __future__ import annotations

import torch

from .moe import MoeLayer, as_bf16, rms_norm


class MoeStack:
    """MoE layers with RMSNorm weights ``norm_weights[L]`` (bf16 [H]) applied to each layer's input."""

    def __init__(self, layers: list, norm_weights: list[torch.Tensor], eps: float = 1e-5, precision: str = "bf16",
                 fuse_router: bool = False):
        if len(norm_weights) != len(layers):
            raise ValueError("one RMSNorm weight per layer")
        self.layers = list(layers)
        dev = self._device()
        self.norm_weights = [as_bf16(w, dev) for w in norm_weights]
        self.eps = float(eps)
        self.precision = precision
        self.fuse_router = bool(fuse_router)
        self._graph = None
        self._static_in = None
        self._static_out = None

    def _device(self) -> torch.device:
        first = self.layers[0]
        return first.device if isinstance(first, MoeLayer) else first.backend.device

    def step(self, hidden: torch.Tensor) -> torch.Tensor:
        """One pass of this rank's tokens bf16 [T, H] through every layer."""
        normed = rms_norm(hidden, self.norm_weights[0], self.eps)
        n = len(self.layers)
        idx = w = None  # routing of this layer, when the previous layer's combine computed it
        for li, layer in enumerate(self.layers):
            last = li + 1 == n
            nxt = None if last else (self.norm_weights[li + 1], self.eps)
            nrouter = None if (last or not self.fuse_router) else self.layers[li + 1]
            ep = not isinstance(layer, MoeLayer)
            if idx is None:
                if last:
                    y, _ = layer.forward(normed, precision=self.precision, residual=hidden)
                elif not ep:
                    y, rb = layer.forward(normed, precision=self.precision, residual=hidden, next_norm=nxt, next_router=nrouter)
                    normed, idx, w = rb.normed, rb.next_indices, rb.next_weights
                else:
                    y, rb, normed = layer.forward(normed, precision=self.precision, residual=hidden, next_norm=nxt,
                                                  next_router=nrouter)
                    idx, w = rb.next_indices, rb.next_weights
            elif last:
                if ep:
                    y, _ = layer.step_routed(normed, idx, w, hidden, None, None, self.precision)
                else:
                    y, _ = layer.experts_forward(normed, idx, w, precision=self.precision, residual=hidden)
            else:
                y, rb = (layer.step_routed(normed, idx, w, hidden, nxt, nrouter, self.precision) if ep
                         else layer.experts_step(normed, idx, w, hidden, nxt, nrouter, self.precision))
                normed, idx, w = rb.normed, rb.next_indices, rb.next_weights
            hidden = y
        return hidden

    def capture(self, example: torch.Tensor, warmup: int = 2) -> None:
        """Record :meth:`step` on a static input buffer shaped like ``example`` as a CUDA graph."""
        self._static_in = example.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):  # workspaces sized and kernels loaded outside the capture
                self.step(self._static_in)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._static_out = self.step(self._static_in)
        self._graph = g

    def replay(self, hidden: torch.Tensor | None = None) -> torch.Tensor:
        """Run the captured step (after copying ``hidden`` into its input buffer); returns its output buffer."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        if hidden is not None:
            self._static_in.copy_(hidden, non_blocking=True)
        self._graph.replay()
        return self._static_out

    def release(self) -> None:
        """Drop the captured graph (before the exchange handles of the layers are closed)."""
        self._graph = None
        self._static_out = None
