"""Expert-parallel layer on GPUs (NCCL), against the single-GPU layer.

Each pair's expert output is computed by the same kernels in both layouts,
and the combine order is the reference's, so the outputs agree (up to the
tile shape the row count selects).  The two-rank test needs two GPUs and is
skipped otherwise.
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


def test_ep_single_rank_matches_layer():
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
        ep = ExpertParallelMoe(0, layer, dev, top_k=4)
        y, rb = ep.forward(x, precision="bf16")
        torch.cuda.synchronize()
        ep.check_device_status()
        assert torch.equal(rb.indices, rb_ref.indices)
        m = parity.assert_output_close(_bits(y), _bits(ref), "ep1 vs layer")
        assert m["bit_equal_frac"] >= 0.99, m
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, q):
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
        ep = ExpertParallelMoe(0, layer, dev, top_k=4)
        for _ in range(2):  # repeated steps reuse the exchange buffers
            y, rb = ep.forward(x, precision="bf16")
            ep.check_device_status()
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(rb.indices, rb_ref.indices)), _bits(y), _bits(ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_match_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
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
