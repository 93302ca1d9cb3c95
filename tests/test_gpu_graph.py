"""One MoE layer call (router, permute, expert GEMMs, combine) captured in a
CUDA graph and replayed: the same results as the eager call, for the captured
input and for new contents of the same input buffer.  Decode at small batch
is launch-bound, so serving loops replay the layer instead of launching its
kernels one by one."""
from __future__ import annotations

import pytest
import torch

from tests.test_gpu_parity import DEV, big_layer  # noqa: F401  (fixture re-export)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 8, 256])
def test_forward_replays_in_cuda_graph(big_layer, T):  # noqa: F811
    from kcapw_klcquant_b200 import synthetic as syn

    x_static = syn.make_hidden(T, 2880, seed=T + 3, device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up off the default stream, as graph capture requires
        for _ in range(2):
            big_layer.forward(x_static)
    torch.cuda.current_stream().wait_stream(side)
    y_ref, rb_ref = big_layer.forward(x_static)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_g, rb_g = big_layer.forward(x_static)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(rb_g.indices, rb_ref.indices) and torch.equal(rb_g.weights, rb_ref.weights)
    assert torch.equal(y_g, y_ref)

    x_new = syn.make_hidden(T, 2880, seed=T + 4, device=DEV)
    x_static.copy_(x_new)
    graph.replay()
    y_new, rb_new = big_layer.forward(x_new)
    torch.cuda.synchronize()
    big_layer.check_device_status()
    assert torch.equal(rb_g.indices, rb_new.indices)
    assert torch.equal(y_g, y_new)

    # a larger eager call allocates a new workspace; the graph keeps the old one
    big_layer.forward(syn.make_hidden(2048, 2880, seed=7, device=DEV))
    y_g.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_g, y_new)
    del graph
