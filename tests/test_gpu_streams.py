"""Reentrancy of the Python layer: calls on different CUDA streams each get a
workspace of their own, so two batches in flight at once give the same bits
as the same calls made one after the other."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("path", ["simt", "tc"])
def test_two_streams_in_flight_match_serial(path):
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    if path not in _lib.capabilities():
        pytest.skip(f"{path} path not built")
    dims = syn.LayerDims(experts=32, hidden=2880, intermediate=2880, top_k=4)
    ml = MoeLayer.from_tensors(0, syn.make_layer(dims, seed=41, device=DEV), DEV, top_k=4, path=path)
    xa = syn.make_hidden(96, dims.hidden, seed=42, device=DEV)
    xb = syn.make_hidden(24, dims.hidden, seed=43, device=DEV)
    ya_ref, ra = ml.forward(xa, precision="bf16")
    yb_ref, rb = ml.forward(xb, precision="bf16")
    ml.check_device_status()
    torch.cuda.synchronize()

    main = torch.cuda.current_stream()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(3):
        s1.wait_stream(main)
        s2.wait_stream(main)
        with torch.cuda.stream(s1):
            ya, _ = ml.forward(xa, precision="bf16")
        with torch.cuda.stream(s2):
            yb, _ = ml.forward(xb, precision="bf16")
        with torch.cuda.stream(s1):
            ya2, _ = ml.forward(xa, precision="bf16")  # s1 again while s2's batch may still run
            ml.check_device_status()  # the status word of s1's own workspace
        torch.cuda.synchronize()
        assert torch.equal(ya, ya_ref) and torch.equal(ya2, ya_ref)
        assert torch.equal(yb, yb_ref)
