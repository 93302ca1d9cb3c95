"""Two-SM expert tiles (klc_set_pair_tiles): a pair of SMs computes two
consecutive 64-row blocks of one expert with one M = 256 block-scaled MMA.

The pair kernel must give the same bits as the one-SM kernel on every row
layout a pair can meet: experts with no rows, with one row, with a half-empty
pair (<= 64 rows), a partial second half, whole pairs, an odd number of 64-row
blocks, in both precisions and with K padded (2880) or not.  The CUDA-core
path (its own arithmetic, checked against the oracle elsewhere) bounds both.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)

# rows per expert: empty, 1, half-empty pairs, partial and whole pairs, odd block counts
COUNTS = [0, 1, 63, 64, 65, 127, 128, 129, 200, 256, 300, 17, 5, 90, 150, 453]


def _routing(counts: list[int], k: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Token slots holding exactly counts[e] pairs of expert e, distinct experts per token."""
    pairs = sum(counts)
    assert pairs % k == 0
    T = pairs // k
    assert max(counts) <= T
    flat = np.repeat(np.arange(len(counts), dtype=np.int32), counts)  # sorted by expert
    idx = np.stack([flat[j * T:(j + 1) * T] for j in range(k)], axis=1)  # token t: flat[t + j*T]
    rng = np.random.default_rng(seed)
    w = rng.random((T, k)).astype(np.float32) + 0.05
    w /= w.sum(axis=1, keepdims=True)
    return torch.from_numpy(idx).to(DEV), torch.from_numpy(w).to(torch.bfloat16).to(DEV)


def _set_mode(mode: int) -> None:
    from kcapw_klcquant_b200 import _lib

    _lib.check(_lib.lib().klc_set_pair_tiles(mode))


@pytest.fixture(autouse=True)
def _restore_default_mode():
    yield
    _set_mode(1)


@pytest.mark.parametrize("hidden,inter", [(2880, 2880), (512, 768)])
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_pair_tiles_match_single_sm_tiles(hidden, inter, precision):
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn
    from tests import parity

    if "tc" not in _lib.capabilities():
        pytest.skip("tensor-core path not built")
    k = 4
    dims = syn.LayerDims(experts=len(COUNTS), hidden=hidden, intermediate=inter, top_k=k)
    ml = MoeLayer.from_tensors(0, syn.make_layer(dims, seed=71, device=DEV), DEV, top_k=k, path="tc")
    idx, w = _routing(COUNTS, k, seed=72)
    x = syn.make_hidden(int(idx.shape[0]), hidden, seed=73, device=DEV)
    res = syn.make_hidden(int(idx.shape[0]), hidden, seed=74, device=DEV)
    outs = {}
    for mode in (0, 2):
        _set_mode(mode)
        y, norms = ml.experts_forward(x, idx, w, precision=precision, return_norms=True, residual=res)
        ml.check_device_status()
        torch.cuda.synchronize()
        outs[mode] = (y.clone(), norms.clone())
    assert torch.equal(outs[0][0], outs[2][0]), "pair tiles changed the layer output"
    # the norms are sums of per-tile partial sums added by float atomics in any order
    torch.testing.assert_close(outs[2][1], outs[0][1], rtol=1e-5, atol=0.0)
    ys, _ = ml.experts_forward(x, idx, w, precision=precision, residual=res, path="simt")
    parity.assert_output_close(outs[2][0].view(torch.int16).cpu().numpy().view(np.uint16),
                               ys.view(torch.int16).cpu().numpy().view(np.uint16), "pair tiles vs CUDA-core path")


def test_pair_tiles_chosen_by_rows_per_expert():
    """Mode 1 (the default) takes the pair kernel at >= 192 rows per expert: the
    router-driven forward gives the same bits in modes 0, 1 and 2."""
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    if "tc" not in _lib.capabilities():
        pytest.skip("tensor-core path not built")
    dims = syn.LayerDims(experts=32, hidden=2880, intermediate=2880, top_k=4)
    ml = MoeLayer.from_tensors(0, syn.make_layer(dims, seed=81, zipf=1.1, device=DEV), DEV, top_k=4)
    x = syn.make_hidden(2048, dims.hidden, seed=82, device=DEV)  # 256 rows per expert on average
    ys = []
    for mode in (0, 1, 2):
        _set_mode(mode)
        y, rb = ml.forward(x, precision="bf16")
        ml.check_device_status()
        torch.cuda.synchronize()
        ys.append(y.clone())
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


@pytest.mark.parametrize("fused_return", [True, False])
def test_pair_tiles_under_expert_parallel_exchange(fused_return):
    """The expert-parallel path (one rank: dispatch into the arena, local expert
    GEMMs on the received rows, return by the down epilogue or by the copy
    kernel, combine) gives the same bits with and without pair tiles, and
    matches the single-GPU layer."""
    import socket

    import torch.distributed as dist

    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe
    from tests import parity

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1, device_id=DEV)
    try:
        dims = syn.LayerDims(32, 2880, 2880, 4)
        layer = syn.make_layer(dims, seed=91, device=DEV)
        x = syn.make_hidden(2048, 2880, seed=92, device=DEV)  # 256 rows per expert on average
        ref, _ = MoeLayer.from_tensors(0, layer, DEV, top_k=4).forward(x, precision="bf16")
        ep = ExpertParallelMoe(0, layer, DEV, top_k=4, exchange="p2p", max_tokens=2048)
        ep._ep.set_fused_return(fused_return)
        ys = {}
        for mode in (0, 2):
            _set_mode(mode)
            for _ in range(2):
                y, _ = ep.forward(x, precision="bf16")
            torch.cuda.synchronize()
            ep.check_device_status()
            ys[mode] = y.clone()
        ep.close()
        assert torch.equal(ys[0], ys[2]), "pair tiles changed the expert-parallel output"
        bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        m = parity.assert_output_close(bits(ys[2]), bits(ref), "ep1 pair tiles vs layer")
        assert m["bit_equal_frac"] >= 0.99, m
    finally:
        dist.destroy_process_group()
