"""The allocation-free entry point klc_moe_experts_noalloc.

It serves callers that cannot allocate device memory themselves (a host
runtime behind an FFI without a CUDA allocator, an application whose device
memory belongs to another pool): instead of a caller workspace it uses a
fixed static device array inside the library.  This file is collected last
so that a run stopping at the first failure has run every other test first;
it also passes on its own in a fresh process (the first call on the device
performs the one-time address lookup).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests import parity

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_noalloc_matches_workspace_entry_point():
    from kcapw_klcquant_b200 import MoeLayer, _lib
    from kcapw_klcquant_b200 import synthetic as syn

    dims = syn.LayerDims(experts=32, hidden=2880, intermediate=2880, top_k=4)
    layer = syn.make_layer(dims, seed=21, device=DEV)
    ml = MoeLayer.from_tensors(0, layer, DEV, top_k=4, path="simt")
    T = 8
    x = syn.make_hidden(T, dims.hidden, seed=21, device=DEV)
    _, rb = ml.forward(x, precision="bf16")
    ref, _ = ml.experts_forward(x, rb.indices, rb.weights, precision="bf16", path="simt")
    torch.cuda.synchronize()

    L = _lib.lib()
    n = ctypes.c_size_t(0)
    _lib.check(L.klc_moe_noalloc_scratch_bytes(ctypes.byref(n)))
    assert 0 < n.value <= 64 << 20
    d = ml.dims(T, "simt")
    for call in range(2):  # the scratch keeps the previous call's contents
        y = torch.full((T, dims.hidden), float("nan"), dtype=torch.bfloat16, device=DEV)
        _lib.check(L.klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(ml.weights), x.data_ptr(), rb.indices.data_ptr(),
                                             rb.weights.data_ptr(), _lib.KLC_PREC_BF16, y.data_ptr(), None, None, _lib.stream_ptr()))
        torch.cuda.synchronize()
        parity.assert_output_close(_bits(y), _bits(ref), f"noalloc call {call}")


def test_noalloc_rejects_oversized_batch():
    from kcapw_klcquant_b200 import _lib

    L = _lib.lib()
    d = _lib.KlcDims(100000, 2880, 2880, 128, 4, _lib.KLC_PATH_SIMT)
    w = _lib.KlcWeights(16, 16, 16, 16, 16, 16, 16, 16, 7.0, 1.702)
    st = L.klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(w), 16, 16, 16, _lib.KLC_PREC_BF16, 16, None, None, None)
    assert st == _lib.KLC_ERR_INVALID
    assert "scratch" in L.klc_last_error().decode()
