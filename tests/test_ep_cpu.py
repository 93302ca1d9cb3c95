"""Expert-parallel exchange logic on CPU ranks (gloo, world size 2 and 4).

The per-rank compute steps are replaced by a CPU backend built on the oracle
(test infrastructure), so these tests check what the GPU path shares with
them: the expert-to-rank partition, the stable packing order, the count and
row exchanges with their split sizes, and the combine of returned rows.  The
result must equal the single-process oracle layer bit for bit.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as orc

E, H, I, K = 16, 64, 64, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class OracleBackend:
    """CPU stand-in for CudaBackend (same method contract)."""

    def __init__(self, layer, lo, hi, top_k):
        p = "model.layers.0.mlp"
        self.rw, self.rb = _bits(layer[f"{p}.router.weight"]), _bits(layer[f"{p}.router.bias"])
        self.top_k = top_k
        self.lo = lo
        e = f"{p}.experts"
        self.ex = orc.DenseExperts(layer[f"{e}.gate_up_proj_blocks"][lo:hi].numpy(), layer[f"{e}.gate_up_proj_scales"][lo:hi].numpy(),
                                   layer[f"{e}.down_proj_blocks"][lo:hi].numpy(), layer[f"{e}.down_proj_scales"][lo:hi].numpy())
        self.gub = _bits(layer[f"{e}.gate_up_proj_bias"][lo:hi])
        self.dnb = _bits(layer[f"{e}.down_proj_bias"][lo:hi])

    def router(self, x):
        lg = orc.router_logits_bits(_bits(x), self.rw, self.rb)
        idx, sc = orc.select_topk(orc.bf16_bits_to_f32(lg), self.top_k)
        return torch.from_numpy(idx), _bf16(orc.softmax_weights_bits(sc))

    def pack(self, idx, x, epr, nranks):
        flat = idx.numpy().reshape(-1).astype(np.int64)
        dest = flat // epr
        order = np.argsort(dest, kind="stable")
        pair_pos = np.empty_like(order)
        pair_pos[order] = np.arange(order.size)
        rows = x[torch.from_numpy(order // idx.shape[1])]
        return (rows.contiguous(), torch.from_numpy((flat % epr)[order].astype(np.int32)),
                torch.from_numpy(np.bincount(dest, minlength=nranks).astype(np.int32)), torch.from_numpy(pair_pos.astype(np.int32)))

    def experts(self, rows, local_ids, precision):
        out = np.zeros((rows.shape[0], rows.shape[1]), np.float32)
        xb = _bits(rows)
        for j, e in enumerate(local_ids.numpy().tolist()):
            gu, dn = self.ex.get(int(e))
            _, _, o = orc.expert_forward(xb[j : j + 1], gu, self.gub[e], dn, self.dnb[e], precision)
            out[j] = o[0]
        return _bf16(orc.f32_to_bf16_bits(out))

    def combine(self, y_rows, pair_pos, w, residual=None):
        T, k = w.shape
        yr = orc.bf16_bits_to_f32(_bits(y_rows))[pair_pos.numpy().reshape(T, k)]
        return _bf16(orc.combine_bits(yr, _bits(w)))


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kcapw_klcquant_b200 import synthetic as syn
        from kcapw_klcquant_b200.ep import ExpertParallelMoe

        layer = syn.make_layer(syn.LayerDims(E, H, I, K), seed=5)
        epr = E // world
        be = OracleBackend(layer, rank * epr, (rank + 1) * epr, K)
        moe = ExpertParallelMoe(0, layer, "cpu", top_k=K, backend=be)
        x = syn.make_hidden(6 + 3 * rank, H, seed=100 + rank)
        y, rb = moe.forward(x, precision="bf16")
        results[rank] = (_bits(y), rb.indices.numpy(), _bits(rb.weights))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    from kcapw_klcquant_b200 import synthetic as syn

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    layer = syn.make_layer(syn.LayerDims(E, H, I, K), seed=5)
    p = "model.layers.0.mlp"
    ex = orc.DenseExperts(*(layer[f"{p}.experts.{n}"].numpy() for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")))
    for rank in range(world):
        y, idx, w = results[rank]
        x = syn.make_hidden(6 + 3 * rank, H, seed=100 + rank)
        ref = orc.moe_layer(_bits(x), idx, w, ex, _bits(layer[f"{p}.experts.gate_up_proj_bias"]), _bits(layer[f"{p}.experts.down_proj_bias"]), "bf16")
        np.testing.assert_array_equal(y, ref)
        # every rank routes over all experts, so remote experts were used
        assert (idx // (E // world) != rank).any()


def test_expert_partition_rejects_uneven_split():
    from kcapw_klcquant_b200.ep import ExpertParallelMoe

    class G:  # a fake 3-rank group for the constructor's arithmetic
        pass

    import unittest.mock as um

    with um.patch("torch.distributed.get_world_size", return_value=3), um.patch("torch.distributed.get_rank", return_value=0):
        with pytest.raises(ValueError):
            ExpertParallelMoe(0, {"model.layers.0.mlp.router.weight": torch.zeros(16, 64)}, "cpu", group=G(), backend=object())


# ---------------------------------------------------------------------------
# failure detection: a rank that dies or stalls must not hang the others
# ---------------------------------------------------------------------------


def _failing_worker(rank, world, port, mode, results):
    """Rank 1 fails (exits, or stalls past the process-group timeout) right before
    the exchange of a forward; the other ranks must get an error, not hang."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe

    layer = syn.make_layer(syn.LayerDims(E, H, I, K), seed=5)
    epr = E // world
    moe = ExpertParallelMoe(0, layer, "cpu", top_k=K, backend=OracleBackend(layer, rank * epr, (rank + 1) * epr, K))
    x = syn.make_hidden(4, H, seed=100 + rank)
    moe.forward(x, precision="bf16")  # one healthy step on every rank
    if rank == 1:
        results[rank] = "failing"
        if mode == "exit":
            os._exit(3)
        time.sleep(40)  # stalls past the peers' timeout; killed by the test afterwards
        os._exit(4)
    t0 = time.monotonic()
    try:
        moe.forward(x, precision="bf16")
        results[rank] = "no error"
    except Exception as e:  # the exchange's collective gives up with an error
        results[rank] = f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_exchange_survivors_get_an_error(mode):
    import time

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    world = 4
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    t0 = time.monotonic()
    survivors = [r for r in range(world) if r != 1]
    for r in survivors:
        procs[r].join(timeout=90)
        assert procs[r].exitcode == 0, f"survivor {r} did not finish cleanly ({procs[r].exitcode})"
    assert time.monotonic() - t0 < 90
    procs[1].join(timeout=1 if mode == "stall" else 30)
    if procs[1].is_alive():
        procs[1].kill()  # the stalled rank (this test's own child process)
        procs[1].join(timeout=10)
    assert results[1] == "failing"
    for r in survivors:
        assert results[r].startswith("error after"), results[r]
