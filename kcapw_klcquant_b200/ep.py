"""Expert-parallel MoE layer: experts sharded over the GPUs of one node.

Experts are sharded contiguously: with N ranks and E experts, rank r holds
the packed MXFP4 weights of experts [r*E/N, (r+1)*E/N) and the replicated
router.  One forward on the rank's own tokens:

1. router (all E experts)                              klc_router_topk
2. dispatch every (token, slot) pair's row to the rank that owns its expert
3. the local experts on the received rows (k = 1)
4. the expert outputs back to the ranks the tokens came from
5. weighted bf16 combine in top-k order                klc_moe_combine

Two exchanges implement steps 2 and 4:

* ``exchange="p2p"`` (default on GPUs): the libklcmoe ``klc_ep_*`` kernels
  store the rows straight into the peers' exchange arenas over NVLink (CUDA
  IPC mappings) and signal each other through flags with bounded waits; the
  whole forward is stream-ordered with no host synchronisation
  (csrc/ep.cu).  The arenas are set up once per layer object by exchanging
  64-byte IPC handles through ``torch.distributed``.
* ``exchange="nccl"``: ``klc_ep_pack`` and ``torch.distributed.all_to_all_single``
  (split sizes read back to the host once per forward).  Any process group
  backend works, so the tests run it on gloo CPU ranks with a CPU backend.

Because every pair's expert output is computed by the same kernels from the
same row, and step 5 is the reference's combine order, the result matches the
single-GPU layer.  The reference has no multi-device path (one process, one
device); this module is new.
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

    def __init__(self, layer_idx: int, tensors: dict[str, torch.Tensor], device, group=None, top_k: int = 4,
                 path: str = "auto", backend=None, share_local: "ExpertParallelMoe | None" = None,
                 exchange: str = "auto", max_tokens: int = 4096, store=None):
        """``tensors`` holds the layer's checkpoint-named tensors: the router and bias
        tensors always, the expert blocks/scales unless ``store`` (an
        :class:`Mxfp4ExpertStore` over the checkpoint) supplies this rank's expert
        shard.  ``share_local``: reuse another instance's resident local experts (same
        expert weights, e.g. the same layer with another router bias).  ``exchange``:
        "p2p", "nccl" or "auto" (p2p for the CUDA backend); ``max_tokens``: the most
        tokens a rank passes to one forward (sizes the p2p exchange arenas)."""
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
        self._ep = None
        self.exchange = "nccl" if backend is not None else ("p2p" if exchange == "auto" else exchange)
        if self.exchange not in ("p2p", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.exchange_name = ("NVLink peer-memory dispatch and combine kernels (libklcmoe klc_ep_*)" if self.exchange == "p2p"
                              else "NCCL all_to_all_single dispatch and combine (split sizes read back to the host)")
        if backend is not None:
            self.backend = backend
            return
        dev = torch.device(device)
        if share_local is not None:
            self.backend = CudaBackend(share_local.backend.local, as_bf16(router_w, dev), as_bf16(tensors[f"{p}.router.bias"], dev),
                                       self.top_k)
            if self.exchange == "p2p":
                self._ep = PeerExchange(self.backend, self.rank, self.world, self.epr, max_tokens, group)
            return
        e = f"{p}.experts"
        if store is not None:
            # this rank's shard read straight from the checkpoint (safetensors slices)
            packed = store.layer(layer_idx, (lo, hi))
        else:
            packed = PackedLayer.from_checkpoint_tensors(
                tensors[f"{e}.gate_up_proj_blocks"][lo:hi], tensors[f"{e}.gate_up_proj_scales"][lo:hi],
                tensors[f"{e}.down_proj_blocks"][lo:hi], tensors[f"{e}.down_proj_scales"][lo:hi], dev,
            )
        local = MoeLayer(packed, router_w[lo:hi], tensors[f"{p}.router.bias"][lo:hi], tensors[f"{e}.gate_up_proj_bias"][lo:hi],
                         tensors[f"{e}.down_proj_bias"][lo:hi], top_k=1, path=path)
        self.backend = CudaBackend(local, as_bf16(router_w, dev), as_bf16(tensors[f"{p}.router.bias"], dev), self.top_k)
        if self.exchange == "p2p":
            self._ep = PeerExchange(self.backend, self.rank, self.world, self.epr, max_tokens, group)

    def _exchange(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]) -> torch.Tensor:
        out = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send, output_split_sizes=recv_counts, input_split_sizes=send_counts, group=self.group)
        return out

    def last_received_rows(self) -> int:
        """(token, expert) pairs this rank's experts processed in the last forward."""
        if self._ep is not None:
            return self._ep.received_rows()
        return int(self._received)

    def check_device_status(self) -> None:
        """Raise if a kernel of the last forward recorded a device-side fault (synchronises)."""
        if self._ep is not None:
            self._ep.check_status()
            return
        local = getattr(self.backend, "local", None)  # host backends have no device status
        if local is not None:
            local.check_device_status()

    def close(self) -> None:
        """Release the p2p exchange arena (collective: every rank calls it; the peers
        must be done writing into it, so the ranks meet at a barrier first)."""
        if self._ep is not None:
            self._ep.close()
            self._ep = None

    def next_router_args(self, T: int) -> tuple:
        """This layer's (replicated) router as the previous layer's fused ``next_router``:
        (klc_next_router, idx, w)."""
        be = self.backend
        dev = be.device
        nidx = torch.empty((T, self.top_k), dtype=torch.int32, device=dev)
        nw = torch.empty((T, self.top_k), dtype=torch.bfloat16, device=dev)
        nr = _lib.KlcNextRouter(be.router_w.data_ptr(), be.router_b.data_ptr(), int(be.router_w.shape[0]), self.top_k,
                                nidx.data_ptr(), nw.data_ptr(), None)
        return nr, nidx, nw

    def step_routed(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor, residual: torch.Tensor,
                    next_norm: tuple[torch.Tensor, float] | None, next_router=None, precision: str = "bf16"):
        """One stacked layer on routing the previous layer computed (p2p exchange):
        dispatch, local experts, combine + residual + the next layer's input RMSNorm
        and, with ``next_router``, its routing of the normalised rows -> (y, RouteBatch)."""
        if self._ep is None:
            raise ValueError("step_routed needs the p2p exchange")
        return self._ep.forward_routed(x, indices, weights, precision, residual, next_norm, next_router)

    def forward(self, x: torch.Tensor, precision: str = "bf16", residual: torch.Tensor | None = None,
                next_norm: tuple[torch.Tensor, float] | None = None, next_router=None):
        """This rank's tokens x bf16 [T, H] -> (y bf16 [T, H], routing); with
        ``next_norm=(weight, eps)`` returns (y, routing, rms_norm(y)) computed by
        the combine kernel (p2p exchange); ``next_router`` (with next_norm) also
        routes rms_norm(y) for the next layer (``routing.next_indices``)."""
        if self._ep is not None:
            if next_router is not None:
                if next_norm is None:
                    raise ValueError("next_router needs next_norm")
                idx, w = self.backend.router(as_bf16(x, self.backend.device))
                y, rb = self._ep.forward_routed(x, idx, w, precision, residual, next_norm, next_router)
                return y, rb, rb.normed
            return self._ep.forward(x, precision, residual, next_norm)
        if next_router is not None:
            raise ValueError("next_router needs the p2p exchange")
        if next_norm is not None:
            raise ValueError("next_norm needs the p2p exchange")
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


class PeerExchange:
    """One rank's side of the NVLink peer-memory exchange (libklcmoe ``klc_ep_*``)."""

    def __init__(self, backend: CudaBackend, rank: int, world: int, experts_per_rank: int, max_tokens: int, group=None):
        self.backend = backend
        self.local = backend.local
        self.device = backend.device
        self.top_k = backend.top_k
        self.group = group
        self.max_tokens = int(max_tokens)
        L = _lib.lib()
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(L.klc_ep_create(rank, world, self.max_tokens, self.top_k, self.local.hidden, experts_per_rank, ctypes.byref(h)))
            self.handle = h
            buf = (ctypes.c_char * 64)()
            _lib.check(L.klc_ep_ipc_handle(h, buf))
            # every rank's arena must have the same layout: same capacity, width, k and expert split
            cfg = torch.tensor([self.max_tokens, self.local.hidden, self.top_k, experts_per_rank], dtype=torch.int64, device=self.device)
            cfgs = torch.empty(world * 4, dtype=torch.int64, device=self.device)
            dist.all_gather_into_tensor(cfgs, cfg, group=group)
            if not bool((cfgs.view(world, 4) == cfg).all()):
                _lib.lib().klc_ep_destroy(h)
                raise ValueError(f"ranks disagree on (max_tokens, hidden, top_k, experts_per_rank): {cfgs.view(world, 4).tolist()}")
            mine = torch.frombuffer(bytearray(bytes(buf)), dtype=torch.uint8).to(self.device)
            everyone = torch.empty(world * 64, dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(everyone, mine, group=group)
            host = bytes(everyone.cpu().numpy().tobytes())
            _lib.check(L.klc_ep_connect(h, host))
            self.dims = _lib.KlcDims(0, self.local.hidden, self.local.intermediate, self.local.experts, 1,
                                     _lib.PATH_CODE[self.local.path])
            n = ctypes.c_size_t(0)
            _lib.check(L.klc_ep_workspace_size(h, ctypes.byref(self.dims), ctypes.byref(n)))
            self.ws = torch.empty(int(n.value), dtype=torch.uint8, device=self.device)
        dist.barrier(group=group)  # every rank connected before any dispatch

    def forward(self, x: torch.Tensor, precision: str = "bf16", residual=None, next_norm=None):
        T, H = int(x.shape[0]), int(x.shape[1])
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange capacity of {self.max_tokens} tokens per rank")
        x = as_bf16(x, self.device)
        dev, k = self.device, self.top_k
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
        slot = torch.empty((T * k,), dtype=torch.int32, device=dev)
        if residual is not None:
            residual = as_bf16(residual, dev)
        norm_w, eps, normed = None, 0.0, None
        if next_norm is not None:
            norm_w, eps = as_bf16(next_norm[0], dev), float(next_norm[1])
            normed = torch.empty_like(out)
        be = self.backend
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().klc_ep_forward(
                self.handle, ctypes.byref(self.dims), ctypes.byref(self.local.weights), be.router_w.data_ptr(), be.router_b.data_ptr(),
                x.data_ptr(), T, _lib.PRECISION_CODE[precision], _lib.ptr(residual), _lib.ptr(norm_w), eps, out.data_ptr(),
                _lib.ptr(normed), idx.data_ptr(), w.data_ptr(), slot.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                _lib.stream_ptr(dev)))
        if next_norm is not None:
            return out, RouteBatch(idx, w, normed=normed), normed
        return out, RouteBatch(idx, w)

    def set_fused_return(self, enabled: bool) -> None:
        """Expert output rows stored to their sources by the down GEMM's epilogue (default) or by a copy kernel."""
        _lib.check(_lib.lib().klc_ep_set_fused_return(self.handle, 1 if enabled else 0))

    def forward_routed(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, precision: str, residual, next_norm,
                       next_router=None):
        """klc_ep_dispatch -> klc_ep_experts -> klc_ep_combine(_route) on given routing."""
        T, H = int(x.shape[0]), int(x.shape[1])
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange capacity of {self.max_tokens} tokens per rank")
        dev = self.device
        x = as_bf16(x, dev)
        idx = idx.to(device=dev, dtype=torch.int32).contiguous()
        w = w.to(device=dev, dtype=torch.bfloat16).contiguous()
        residual = as_bf16(residual, dev) if residual is not None else None
        if next_norm is None and next_router is not None:
            raise ValueError("next_router needs next_norm")
        norm_w, eps = (as_bf16(next_norm[0], dev), float(next_norm[1])) if next_norm is not None else (None, 0.0)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        normed = torch.empty_like(out) if next_norm is not None else None
        slot = torch.empty((T * self.top_k,), dtype=torch.int32, device=dev)
        L = _lib.lib()
        s = _lib.stream_ptr(dev)
        nidx = nw = None
        with torch.cuda.device(dev):
            _lib.check(L.klc_ep_dispatch(self.handle, idx.data_ptr(), T, x.data_ptr(), slot.data_ptr(), self.ws.data_ptr(),
                                         self.ws.numel(), s))
            _lib.check(L.klc_ep_experts(self.handle, ctypes.byref(self.dims), ctypes.byref(self.local.weights),
                                        _lib.PRECISION_CODE[precision], self.ws.data_ptr(), self.ws.numel(), s))
            if next_router is not None:
                nr, nidx, nw = next_router.next_router_args(T)
                _lib.check(L.klc_ep_combine_route(self.handle, slot.data_ptr(), w.data_ptr(), T, _lib.ptr(residual),
                                                  norm_w.data_ptr(), eps, out.data_ptr(), normed.data_ptr(), ctypes.byref(nr), s))
            else:
                _lib.check(L.klc_ep_combine(self.handle, slot.data_ptr(), w.data_ptr(), T, _lib.ptr(residual), _lib.ptr(norm_w),
                                            eps, out.data_ptr(), _lib.ptr(normed), s))
        return out, RouteBatch(idx, w, normed=normed, next_indices=nidx, next_weights=nw)

    def received_rows(self) -> int:
        n = ctypes.c_int64(0)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().klc_ep_received_rows(self.handle, ctypes.byref(n), _lib.stream_ptr(self.device)))
        return int(n.value)

    def check_status(self) -> None:
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().klc_ep_status(self.handle, self.ws.data_ptr(), None, None, _lib.stream_ptr(self.device)))

    def close(self) -> None:
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        _lib.check(_lib.lib().klc_ep_destroy(self.handle))
        self.handle = None
