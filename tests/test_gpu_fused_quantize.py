"""The down operand quantized inside the gate_up epilogue (klc_set_fused_quantize)
against the separate quantize pass over the bf16 gated rows: the layer output
must be the same bits for 16-row, 64-row and two-SM tiles, both precisions,
padded and unpadded K, and rows that end mid-tile."""
from __future__ import annotations

import pytest
import torch

from tests.test_gpu_pair_tiles import COUNTS, DEV, _routing, _set_mode

pytestmark = pytest.mark.gpu


def _set_fused(enable: bool) -> None:
    from kcapw_klcquant_b200 import _lib

    _lib.check(_lib.lib().klc_set_fused_quantize(1 if enable else 0))


@pytest.fixture(autouse=True)
def _restore_defaults():
    yield
    _set_fused(True)
    _set_mode(1)


def _both(fn):
    outs = []
    for fused in (False, True):
        _set_fused(fused)
        y, norms = fn()
        torch.cuda.synchronize()
        outs.append((y.clone(), None if norms is None else norms.clone()))
    return outs


@pytest.mark.parametrize("hidden,inter", [(2880, 2880), (512, 768)])
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("pair_mode", [0, 2])
def test_fused_quantize_matches_separate_pass(hidden, inter, precision, pair_mode):
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    if "tc" not in _lib.capabilities():
        pytest.skip("tensor-core path not built")
    _set_mode(pair_mode)
    k = 4
    dims = syn.LayerDims(experts=len(COUNTS), hidden=hidden, intermediate=inter, top_k=k)
    ml = MoeLayer.from_tensors(0, syn.make_layer(dims, seed=101, device=DEV), DEV, top_k=k, path="tc")
    idx, w = _routing(COUNTS, k, seed=102)
    x = syn.make_hidden(int(idx.shape[0]), hidden, seed=103, device=DEV)
    (y0, n0), (y1, n1) = _both(lambda: ml.experts_forward(x, idx, w, precision=precision, return_norms=True))
    ml.check_device_status()
    assert torch.equal(y0, y1), "the fused quantize changed the layer output"
    torch.testing.assert_close(n1, n0, rtol=1e-5, atol=0.0)  # float-atomic sums in another order


@pytest.mark.parametrize("tokens", [1, 7, 256])
def test_fused_quantize_decode_tiles(tokens):
    """16-row tiles (decode: a few rows per expert) keep the separate pass: the
    switch leaves the routed forward unchanged."""
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    if "tc" not in _lib.capabilities():
        pytest.skip("tensor-core path not built")
    dims = syn.LayerDims(experts=128, hidden=2880, intermediate=2880, top_k=4)
    ml = MoeLayer.from_tensors(0, syn.make_layer(dims, seed=111, device=DEV), DEV, top_k=4)
    x = syn.make_hidden(tokens, 2880, seed=112, device=DEV)
    (y0, _), (y1, _) = _both(lambda: (ml.forward(x, precision="bf16")[0], None))
    ml.check_device_status()
    assert torch.equal(y0, y1)
