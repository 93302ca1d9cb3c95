"""Expert-parallel layer on GPUs against the single-GPU layer, for both
exchanges: the NVLink peer-memory kernels (``p2p``, libklcmoe klc_ep_*) and
NCCL all_to_all_single (``nccl``).

Each pair's expert output is computed by the same kernels in both layouts,
and the combine order is the reference's, so the outputs agree (up to the
tile shape the row count selects).  The two-rank test needs two GPUs and is
skipped otherwise.  The exchange's bounded waits are checked on one GPU with
a peer that never signals.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import parity

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_ep_single_rank_matches_layer(exchange):
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe

    dev = torch.device("cuda", 0)
    port = _free_port()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1, device_id=dev)
    try:
        dims = syn.LayerDims(32, 2880, 2880, 4)
        layer = syn.make_layer(dims, seed=7, device=dev)
        x = syn.make_hidden(64, 2880, seed=7, device=dev)
        ref, rb_ref = MoeLayer.from_tensors(0, layer, dev, top_k=4).forward(x, precision="bf16")
        ep = ExpertParallelMoe(0, layer, dev, top_k=4, exchange=exchange, max_tokens=64)
        for _ in range(3):  # repeated steps reuse the exchange buffers
            y, rb = ep.forward(x, precision="bf16")
        torch.cuda.synchronize()
        ep.check_device_status()
        assert torch.equal(rb.indices, rb_ref.indices)
        if exchange == "p2p":
            # rows returned by the copy kernel instead of the down epilogue: identical output
            ep._ep.set_fused_return(False)
            y_copy, _ = ep.forward(x, precision="bf16")
            ep._ep.set_fused_return(True)
            ep.check_device_status()
            assert torch.equal(y_copy, y)
        m = parity.assert_output_close(_bits(y), _bits(ref), f"ep1 ({exchange}) vs layer")
        assert m["bit_equal_frac"] >= 0.99, m
        if exchange == "p2p":
            # residual + the next layer's RMSNorm fused into the exchange's combine
            res = syn.make_hidden(64, 2880, seed=8, device=dev)
            nw = syn.make_rms_weight(2880, seed=8, device=dev)
            y2, _, normed = ep.forward(x, precision="bf16", residual=res, next_norm=(nw, 1e-5))
            ref2, rb2 = MoeLayer.from_tensors(0, layer, dev, top_k=4).forward(x, precision="bf16", residual=res, next_norm=(nw, 1e-5))
            parity.assert_output_close(_bits(y2), _bits(ref2), "ep1 residual")
            parity.assert_output_close(_bits(normed), _bits(rb2.normed), "ep1 normed")
            ep.check_device_status()
        ep.close()
    finally:
        dist.destroy_process_group()


def test_ep_wait_expires_without_peer():
    """A rank whose peer never signals: the exchange's bounded waits give up,
    record KLC_ERR_DEVICE_TIMEOUT (site 100 + the silent rank) and return; the
    GPU keeps answering.  Both ranks' IPC handles are this process's own arena,
    so every store stays inside it; nothing ever raises rank 1's flags."""
    import ctypes

    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    E, H, epr, T = 16, 256, 8, 24
    layer = syn.make_layer(syn.LayerDims(E, H, H, 4), seed=9, device=dev)
    p = "model.layers.0.mlp"
    e = f"{p}.experts"
    from kcapw_klcquant_b200.mxfp4_expert import PackedLayer

    packed = PackedLayer.from_checkpoint_tensors(layer[f"{e}.gate_up_proj_blocks"][:epr], layer[f"{e}.gate_up_proj_scales"][:epr],
                                                 layer[f"{e}.down_proj_blocks"][:epr], layer[f"{e}.down_proj_scales"][:epr], dev)
    local = MoeLayer(packed, layer[f"{p}.router.weight"][:epr], layer[f"{p}.router.bias"][:epr], layer[f"{e}.gate_up_proj_bias"][:epr],
                     layer[f"{e}.down_proj_bias"][:epr], top_k=1, path="simt")
    h = ctypes.c_void_p()
    _lib.check(L.klc_ep_create(0, 2, T, 4, H, epr, ctypes.byref(h)))
    try:
        _lib.check(L.klc_ep_set_wait_limit_ns(h, 50_000_000))  # 50 ms
        buf = (ctypes.c_char * 64)()
        _lib.check(L.klc_ep_ipc_handle(h, buf))
        _lib.check(L.klc_ep_connect(h, bytes(buf) * 2))
        dims = _lib.KlcDims(0, H, H, epr, 1, _lib.KLC_PATH_SIMT)
        n = ctypes.c_size_t(0)
        _lib.check(L.klc_ep_workspace_size(h, ctypes.byref(dims), ctypes.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
        x = syn.make_hidden(T, H, seed=9, device=dev)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        idx = torch.empty((T, 4), dtype=torch.int32, device=dev)
        w = torch.empty((T, 4), dtype=torch.bfloat16, device=dev)
        slot = torch.empty((T * 4,), dtype=torch.int32, device=dev)
        rw, rb = layer[f"{p}.router.weight"].contiguous(), layer[f"{p}.router.bias"].contiguous()
        _lib.check(L.klc_ep_forward(h, ctypes.byref(dims), ctypes.byref(local.weights), rw.data_ptr(), rb.data_ptr(), x.data_ptr(), T,
                                    _lib.KLC_PREC_BF16, None, None, 0.0, out.data_ptr(), None, idx.data_ptr(), w.data_ptr(),
                                    slot.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr()))
        code, where = ctypes.c_int(0), ctypes.c_int(0)
        st = L.klc_ep_status(h, ws.data_ptr(), ctypes.byref(code), ctypes.byref(where), _lib.stream_ptr())
        assert st == _lib.KLC_ERR_DEVICE_TIMEOUT and code.value == _lib.KLC_ERR_DEVICE_TIMEOUT, (st, code.value, where.value)
        assert where.value in (101, 301), where.value
        assert float(torch.ones(4, device=dev).sum()) == 4.0  # the context is still usable
    finally:
        L.klc_ep_destroy(h)


def _worker(rank, world, port, q, exchange):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world, device_id=dev)
    try:
        from kcapw_klcquant_b200 import MoeLayer
        from kcapw_klcquant_b200 import synthetic as syn
        from kcapw_klcquant_b200.ep import ExpertParallelMoe

        layer = syn.make_layer(syn.GPT_OSS_120B, seed=3, device=dev)
        x = syn.make_hidden(96 + 32 * rank, 2880, seed=50 + rank, device=dev)
        ref, rb_ref = MoeLayer.from_tensors(0, layer, dev, top_k=4).forward(x, precision="bf16")
        ep = ExpertParallelMoe(0, layer, dev, top_k=4, exchange=exchange, max_tokens=256)
        for _ in range(3):  # repeated steps reuse the exchange buffers
            y, rb = ep.forward(x, precision="bf16")
            ep.check_device_status()
        same_copy = True
        if exchange == "p2p":
            # rows returned by a copy kernel instead of the down epilogue's peer stores: same bits
            ep._ep.set_fused_return(False)
            y_copy, _ = ep.forward(x, precision="bf16")
            ep.check_device_status()
            ep._ep.set_fused_return(True)
            y_again, _ = ep.forward(x, precision="bf16")
            ep.check_device_status()
            same_copy = bool(torch.equal(y_copy, y)) and bool(torch.equal(y_again, y))
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(rb.indices, rb_ref.indices)) and same_copy, _bits(y), _bits(ref)))
        ep.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_ep_two_ranks_match_single_gpu(exchange):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_route, y, ref in out:
        assert same_route
        m = parity.assert_output_close(y, ref, f"ep2 rank {rank}")
        assert m["bit_equal_frac"] >= 0.99, m


def test_ep_from_checkpoint_store_and_stack(tmp_path):
    """The rank's expert shard read from a safetensors checkpoint (Mxfp4ExpertStore
    with expert_range) gives the same layer as the in-memory tensors; a two-layer
    MoeStack (RMSNorm + residual between the blocks) over it, eager and as a
    captured CUDA graph, equals the single-GPU layers."""
    import json

    from safetensors.torch import save_file

    from kcapw_klcquant_b200 import MoeLayer, Mxfp4ExpertStore
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe
    from kcapw_klcquant_b200.stack import MoeStack

    dev = torch.device("cuda", 0)
    dims = syn.LayerDims(16, 2880, 2880, 4)
    layers = {li: syn.make_layer(dims, seed=60 + li, layer_idx=li) for li in range(2)}
    experts = {k: v.contiguous() for t in layers.values() for k, v in t.items() if ".experts." in k and (k.endswith("_blocks") or k.endswith("_scales"))}
    save_file(experts, str(tmp_path / "model-00000.safetensors"))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {k: "model-00000.safetensors" for k in experts}}))
    store = Mxfp4ExpertStore(tmp_path, tmp_path, dev, dtype=torch.bfloat16)
    port = _free_port()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1, device_id=dev)
    try:
        dense = {li: {k: v.to(dev) for k, v in syn.dense_tensors(t, li).items()} for li, t in layers.items()}
        eps = [ExpertParallelMoe(li, dense[li], dev, top_k=4, store=store, max_tokens=16) for li in range(2)]
        assert store.resident_experts(0) == set(range(16))
        singles = [MoeLayer.from_tensors(li, {k: v.to(dev) for k, v in layers[li].items()}, dev, top_k=4) for li in range(2)]
        norms = [syn.make_rms_weight(2880, seed=70 + li, device=dev) for li in range(2)]
        x = syn.make_hidden(16, 2880, seed=61, device=dev)
        ref = MoeStack(singles, norms).step(x)
        st = MoeStack(eps, norms)
        y = st.step(x)
        parity.assert_output_close(_bits(y), _bits(ref), "stack from store")
        assert float(torch.mean((y.view(torch.int16) == ref.view(torch.int16)).float())) >= 0.99
        st.capture(x)
        for _ in range(2):  # replays advance the exchange epochs on the device
            yg = st.replay(x).clone()
            torch.cuda.synchronize()
            assert torch.equal(yg, y)
        for ep in eps:
            ep.check_device_status()
        st.release()
        for ep in eps:
            ep.close()
    finally:
        dist.destroy_process_group()
