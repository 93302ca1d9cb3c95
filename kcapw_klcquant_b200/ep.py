"""Expert-parallel MoE layer over torch.distributed (NCCL on GPUs).

Experts are sharded contiguously: with N ranks and E experts, rank r holds
the packed MXFP4 weights of experts [r*E/N, (r+1)*E/N) and the replicated
router.  One forward on the rank's own tokens:

1. router (all E experts)                      klc_router_topk
2. pack (token, slot) pairs by owning rank      klc_ep_pack (stable counting sort + row gather)
3. exchange pair counts, then token rows and    all_to_all_single (NCCL)
   local expert ids
4. run the received rows through the local      klc_moe_experts with k = 1, weight 1.0
   experts (y = out.to(bf16) of each pair)
5. send the expert outputs back                 all_to_all_single (reverse splits)
6. weighted bf16 combine in top-k order         klc_moe_combine

Because every pair's expert output is computed by the same kernels from the
same row and weights, and step 6 is the reference's combine order, the
result matches the single-GPU layer.  The reference has no multi-device
path (it runs one process on one device); this module is new.

The per-rank compute steps are methods of a backend object, so the
exchange logic can be exercised with CPU ranks (gloo) and a CPU backend in
the tests; the product uses :class:`CudaBackend` (libklcmoe.so kernels).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .moe import MoeLayer, RouteBatch, as_bf16, workspace
from .mxfp4_expert import PackedLayer


class CudaBackend:
    """Per-rank compute on the GPU through libklcmoe.so."""

    def __init__(self, local: MoeLayer, router_w: torch.Tensor, router_b: torch.Tensor, top_k: int):
        self.local = local
        self.router_w = router_w
        self.router_b = router_b
        self.top_k = top_k
        self.device = local.device

    def router(self, x: torch.Tensor):
        T, H = x.shape
        E = int(self.router_w.shape[0])
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, self.top_k), dtype=torch.bfloat16, device=self.device)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().klc_router_topk(x.data_ptr(), T, H, self.router_w.data_ptr(), self.router_b.data_ptr(), E,
                                                  self.top_k, None, idx.data_ptr(), w.data_ptr(), None, _lib.stream_ptr()))
        return idx, w

    def pack(self, idx: torch.Tensor, x: torch.Tensor, experts_per_rank: int, nranks: int):
        T, H = x.shape
        k = int(idx.shape[1])
        send_rows = torch.empty((T * k, H), dtype=torch.bfloat16, device=self.device)
        send_expert = torch.empty((T * k,), dtype=torch.int32, device=self.device)
        send_counts = torch.empty((nranks,), dtype=torch.int32, device=self.device)
        pair_pos = torch.empty((T * k,), dtype=torch.int32, device=self.device)
        dims = _lib.KlcDims(T, 64, 64, max(nranks, k), k, _lib.KLC_PATH_SIMT)
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().klc_moe_workspace_size(ctypes.byref(dims), ctypes.byref(n)))
        ws = workspace(self.device, n.value)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().klc_ep_pack(idx.data_ptr(), T, k, experts_per_rank, nranks, x.data_ptr(), H,
                                              send_rows.data_ptr(), send_expert.data_ptr(), send_counts.data_ptr(),
                                              pair_pos.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr()))
        return send_rows, send_expert, send_counts, pair_pos

    def experts(self, rows: torch.Tensor, local_ids: torch.Tensor, precision: str) -> torch.Tensor:
        R = int(rows.shape[0])
        if R == 0:
            return torch.empty((0, self.local.hidden), dtype=torch.bfloat16, device=self.device)
        ones = torch.ones((R, 1), dtype=torch.bfloat16, device=self.device)
        y, _ = self.local.experts_forward(rows, local_ids.reshape(R, 1), ones, precision=precision)
        return y

    def combine(self, y_rows: torch.Tensor, pair_pos: torch.Tensor, w: torch.Tensor, residual=None,
                next_norm=None) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
        """Weighted combine of the returned rows; with ``next_norm=(weight, eps)`` also the RMSNorm of the result."""
        T, k = w.shape
        H = int(y_rows.shape[1])
        out = torch.empty((T, H), dtype=torch.bfloat16, device=self.device)
        with torch.cuda.device(self.device):
            if next_norm is None:
                _lib.check(_lib.lib().klc_moe_combine(y_rows.data_ptr(), pair_pos.data_ptr(), w.data_ptr(), T, k, H,
                                                      _lib.ptr(residual), out.data_ptr(), _lib.stream_ptr()))
                return out
            norm_w = next_norm[0].to(device=self.device, dtype=torch.bfloat16).contiguous()
            normed = torch.empty_like(out)
            _lib.check(_lib.lib().klc_moe_combine_rmsnorm(y_rows.data_ptr(), pair_pos.data_ptr(), w.data_ptr(), T, k, H,
                                                          _lib.ptr(residual), norm_w.data_ptr(), float(next_norm[1]),
                                                          out.data_ptr(), normed.data_ptr(), _lib.stream_ptr()))
        return out, normed


def _rows_as_bytes(t: torch.Tensor) -> torch.Tensor:
    """[R, H] 2-byte rows viewed as [R, 2H] uint8 (every backend moves bytes)."""
    return t.contiguous().view(torch.uint8).reshape(t.shape[0], -1)


class ExpertParallelMoe:
    """One MoE layer sharded over the ranks of ``group`` (E divisible by the world size)."""

    exchange_name = "NCCL all_to_all_single dispatch and combine (split sizes synchronised through the host)"

    def __init__(self, layer_idx: int, tensors: dict[str, torch.Tensor], device, group=None, top_k: int = 4,
                 path: str = "auto", backend=None, share_local: "ExpertParallelMoe | None" = None):
        """``share_local``: reuse another instance's resident local experts (same expert
        weights, e.g. the same layer with another router bias)."""
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.top_k = int(top_k)
        p = f"model.layers.{layer_idx}.mlp"
        router_w = tensors[f"{p}.router.weight"]
        E = int(router_w.shape[0])
        if E % self.world:
            raise ValueError(f"{E} experts cannot be split evenly over {self.world} ranks")
        self.experts = E
        self.epr = E // self.world
        lo, hi = self.rank * self.epr, (self.rank + 1) * self.epr
        self.local_range = (lo, hi)
        self._received = 0
        if backend is not None:
            self.backend = backend
            return
        dev = torch.device(device)
        if share_local is not None:
            self.backend = CudaBackend(share_local.backend.local, as_bf16(router_w, dev), as_bf16(tensors[f"{p}.router.bias"], dev),
                                       self.top_k)
            return
        e = f"{p}.experts"
        packed = PackedLayer.from_checkpoint_tensors(
            tensors[f"{e}.gate_up_proj_blocks"][lo:hi], tensors[f"{e}.gate_up_proj_scales"][lo:hi],
            tensors[f"{e}.down_proj_blocks"][lo:hi], tensors[f"{e}.down_proj_scales"][lo:hi], dev,
        )
        local = MoeLayer(packed, router_w[lo:hi], tensors[f"{p}.router.bias"][lo:hi], tensors[f"{e}.gate_up_proj_bias"][lo:hi],
                         tensors[f"{e}.down_proj_bias"][lo:hi], top_k=1, path=path)
        self.backend = CudaBackend(local, as_bf16(router_w, dev), as_bf16(tensors[f"{p}.router.bias"], dev), self.top_k)

    def _exchange(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]) -> torch.Tensor:
        out = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send, output_split_sizes=recv_counts, input_split_sizes=send_counts, group=self.group)
        return out

    def last_received_rows(self) -> int:
        """(token, expert) pairs this rank's experts processed in the last forward."""
        return int(self._received)

    def check_device_status(self) -> None:
        """Raise if a kernel of the last local expert call recorded a device-side fault (synchronises)."""
        local = getattr(self.backend, "local", None)  # host backends have no device status
        if local is not None:
            local.check_device_status()

    def forward(self, x: torch.Tensor, precision: str = "bf16", residual: torch.Tensor | None = None) -> tuple[torch.Tensor, RouteBatch]:
        be = self.backend
        idx, w = be.router(x)
        send_rows, send_expert, send_counts, pair_pos = be.pack(idx, x, self.epr, self.world)
        recv_counts_t = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts_t, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts_t]).cpu()  # one host sync for both split lists
        sc, rc = counts[0].tolist(), counts[1].tolist()
        self._received = sum(rc)
        recv_rows = self._exchange(_rows_as_bytes(send_rows), sc, rc).view(send_rows.dtype).reshape(-1, send_rows.shape[1])
        recv_expert = self._exchange(send_expert, sc, rc)
        y_local = be.experts(recv_rows, recv_expert, precision)
        y_back = self._exchange(_rows_as_bytes(y_local), rc, sc).view(y_local.dtype).reshape(-1, y_local.shape[1])
        out = be.combine(y_back, pair_pos, w, residual)
        return out, RouteBatch(idx, w)
