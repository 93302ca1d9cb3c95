"""The allocation-free entry point klc_moe_experts_noalloc.

Some callers of this library cannot allocate device memory where they run the
MoE layer: a host runtime that reaches the C ABI through a foreign-function
interface and has no CUDA allocator of its own, or an application whose device
memory all belongs to another pool.  For them the library offers an entry
point whose scratch is a fixed static device array inside the library instead
of a caller workspace.

These tests call it through the C ABI and require its output to be
bit-identical to klc_moe_experts on the CUDA-core path (both run the same
kernels in the same order), and within the stated tolerance of the CPU oracle.
Two calls run back to back, the second smaller than the first, so stale
contents of the shared array cannot leak into a result.  This file is collected
last so that a run stopping at the first failure has run every other test; it
also passes alone in a fresh process, where its first call performs the
one-time address lookup.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests import parity

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
E, H, I, K = 32, 2880, 2880, 4


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def setup():
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn

    dims = syn.LayerDims(experts=E, hidden=H, intermediate=I, top_k=K)
    layer = syn.make_layer(dims, seed=21)
    ml = MoeLayer.from_tensors(0, layer, DEV, top_k=K, path="simt")
    return layer, ml


def _noalloc(ml, x, idx, w, norms, residual):
    from kcapw_klcquant_b200 import _lib

    T = int(x.shape[0])
    d = ml.dims(T, "simt")
    y = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(ml.weights), x.data_ptr(), idx.data_ptr(),
                                                  w.data_ptr(), _lib.KLC_PREC_BF16, y.data_ptr(), _lib.ptr(norms),
                                                  _lib.ptr(residual), _lib.stream_ptr()))
    torch.cuda.synchronize()
    assert _lib.lib().klc_moe_noalloc_status(None, None, None, _lib.stream_ptr()) == _lib.KLC_OK
    return y


@pytest.mark.parametrize("with_norms", [False, True])
@pytest.mark.parametrize("with_residual", [False, True])
def test_noalloc_matches_workspace_entry_point(setup, with_norms, with_residual):
    from kcapw_klcquant_b200 import _lib
    from kcapw_klcquant_b200 import synthetic as syn

    layer, ml = setup
    n = ctypes.c_size_t(0)
    _lib.check(_lib.lib().klc_moe_noalloc_scratch_bytes(ctypes.byref(n)))
    assert 0 < n.value <= 64 << 20
    p = "model.layers.0.mlp"
    ex = orc.DenseExperts(*(layer[f"{p}.experts.{k}"].numpy() for k in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")), max_cached=1)
    gub, dnb = _bits(layer[f"{p}.experts.gate_up_proj_bias"]), _bits(layer[f"{p}.experts.down_proj_bias"])
    # a larger call, then a smaller one: the shared array still holds the first call's contents
    for call, T in enumerate((32, 8)):
        x = syn.make_hidden(T, H, seed=100 + T, device=DEV)
        _, rb = ml.forward(x, precision="bf16")
        residual = syn.make_hidden(T, H, seed=200 + T, device=DEV) if with_residual else None
        ref, ref_norms = ml.experts_forward(x, rb.indices, rb.weights, precision="bf16", return_norms=with_norms,
                                            residual=residual, path="simt")
        norms = torch.full((T, K, 2), float("nan"), dtype=torch.float32, device=DEV) if with_norms else None
        y = _noalloc(ml, x, rb.indices, rb.weights, norms, residual)
        np.testing.assert_array_equal(_bits(y), _bits(ref), err_msg=f"noalloc call {call} (T={T})")
        if with_norms:
            np.testing.assert_allclose(norms.cpu().numpy(), ref_norms.cpu().numpy(), rtol=1e-5)
        if call == 1 and not with_residual:
            # and within the tolerance of the CPU oracle of the reference's bf16 path
            want = orc.moe_layer(_bits(x), rb.indices.cpu().numpy(), _bits(rb.weights), ex, gub, dnb, "bf16")
            parity.assert_output_close(_bits(y), want, f"noalloc vs oracle T={T}")


def test_noalloc_reports_bad_expert_index(setup):
    from kcapw_klcquant_b200 import _lib
    from kcapw_klcquant_b200 import synthetic as syn

    _, ml = setup
    T = 4
    x = syn.make_hidden(T, H, seed=7, device=DEV)
    idx = torch.tensor([[0, 1, 2, 3], [4, E + 5, 6, 7], [8, 9, 10, 11], [12, 13, 14, 15]], dtype=torch.int32, device=DEV)
    w = torch.full((T, K), 0.25, dtype=torch.bfloat16, device=DEV)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
    d = ml.dims(T, "simt")
    _lib.check(_lib.lib().klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(ml.weights), x.data_ptr(), idx.data_ptr(),
                                                  w.data_ptr(), _lib.KLC_PREC_BF16, y.data_ptr(), None, None, _lib.stream_ptr()))
    code = ctypes.c_int(0)
    st = _lib.lib().klc_moe_noalloc_status(ctypes.byref(code), None, None, _lib.stream_ptr())
    assert st == _lib.KLC_ERR_DEVICE_FAULT and code.value == _lib.KLC_ERR_DEVICE_FAULT
    # the next good call clears the status word
    idx_ok = torch.arange(T * K, dtype=torch.int32, device=DEV).reshape(T, K) % E
    _noalloc(ml, x, idx_ok, w, None, None)


def test_noalloc_rejects_oversized_batch():
    from kcapw_klcquant_b200 import _lib

    L = _lib.lib()
    d = _lib.KlcDims(100000, 2880, 2880, 128, 4, _lib.KLC_PATH_SIMT)
    w = _lib.KlcWeights(16, 16, 16, 16, 16, 16, 16, 16, 7.0, 1.702)
    st = L.klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(w), 16, 16, 16, _lib.KLC_PREC_BF16, 16, None, None, None)
    assert st == _lib.KLC_ERR_INVALID
    assert "scratch" in L.klc_last_error().decode()
