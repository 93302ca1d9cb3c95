"""The combine fused with the residual add and the next layer's input RMSNorm
(klc_moe_combine_rmsnorm, klc_moe_forward_rmsnorm) against the oracle.

The executor adds the MoE output to the residual stream
(streamed_transformer_executor.py:260) and the next layer starts with
rms_norm(hidden, input_layernorm.weight) (:235, streamed_attention.py:27-28).
The residual sum is bit-exact (bf16 arithmetic in a fixed order); the norm
sums squares in a different order than torch, so it is held to the
standalone RMSNorm's tolerance: at most 1 bf16 ulp, on under 1 % of values.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests import parity
from tests.test_gpu_parity import DEV, PATHS, bits_of, case_cache, load  # noqa: F401  (fixture re-export)

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    return orc.f32_to_bf16_bits(np.asarray(a, dtype=np.float32))


def _dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def _residual_add_bits(acc_bits: np.ndarray, res_bits: np.ndarray) -> np.ndarray:
    return orc.f32_to_bf16_bits(orc.round_bf16(orc.bf16_bits_to_f32(res_bits) + orc.bf16_bits_to_f32(acc_bits)))


def _check_norm(got_bits: np.ndarray, want_bits: np.ndarray) -> None:
    d = parity.ulp_distance_bf16(got_bits, want_bits)
    assert d.max() <= 1 and np.mean(d > 0) < 0.01, (int(d.max()), float(np.mean(d > 0)))


@pytest.mark.parametrize("with_residual", [False, True])
@pytest.mark.parametrize("T,k,H", [(1, 4, 2880), (37, 4, 2880), (16, 1, 128), (9, 8, 64), (300, 4, 2880)])
def test_combine_rmsnorm_vs_oracle(T, k, H, with_residual):
    from kcapw_klcquant_b200 import _lib, rms_norm

    rng = np.random.default_rng(T * 131 + k * 7 + H + with_residual)
    R = T * k + 5  # a few rows that no pair reads
    y_bits = _bf16_bits(rng.standard_normal((R, H)) * 2.0)
    pair_pos = rng.permutation(R)[: T * k].astype(np.int32)
    w_bits = _bf16_bits(rng.random((T, k)) / k)
    res_bits = _bf16_bits(rng.standard_normal((T, H)) * 4.0) if with_residual else None
    g_bits = _bf16_bits(1.0 + 0.1 * rng.standard_normal(H))

    y, pp, w, g = _dev(y_bits), torch.from_numpy(pair_pos).to(DEV), _dev(w_bits), _dev(g_bits)
    res = _dev(res_bits) if with_residual else None
    out = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
    normed = torch.empty_like(out)
    out_plain = torch.empty_like(out)
    L = _lib.lib()
    with torch.cuda.device(DEV):
        _lib.check(L.klc_moe_combine_rmsnorm(y.data_ptr(), pp.data_ptr(), w.data_ptr(), T, k, H, _lib.ptr(res),
                                             g.data_ptr(), EPS, out.data_ptr(), normed.data_ptr(), _lib.stream_ptr()))
        _lib.check(L.klc_moe_combine(y.data_ptr(), pp.data_ptr(), w.data_ptr(), T, k, H, _lib.ptr(res),
                                     out_plain.data_ptr(), _lib.stream_ptr()))
    torch.cuda.synchronize()

    rows = orc.bf16_bits_to_f32(y_bits)[pair_pos].reshape(T, k, H)
    want_out = orc.combine_bits(rows, w_bits)
    if with_residual:
        want_out = _residual_add_bits(want_out, res_bits)
    got_out = bits_of(out)
    assert np.array_equal(got_out, want_out)
    assert np.array_equal(got_out, bits_of(out_plain))  # the fused form stores the same residual sum
    _check_norm(bits_of(normed), orc.rms_norm_bits(want_out, g_bits, EPS))
    _check_norm(bits_of(normed), bits_of(rms_norm(out, g, EPS)))


@pytest.mark.parametrize("path", PATHS)
def test_forward_next_norm(case_cache, path):  # noqa: F811
    fx, dims, layer, x, ml = load(case_cache, "mini_e16_h256_t32")
    rng = np.random.default_rng(5)
    H = ml.hidden
    res = _dev(_bf16_bits(rng.standard_normal((x.shape[0], H))))
    g = _dev(_bf16_bits(1.0 + 0.1 * rng.standard_normal(H)))
    y0, rb0 = ml.forward(x.to(DEV), precision="bf16", residual=res, path=path)
    y1, rb1 = ml.forward(x.to(DEV), precision="bf16", residual=res, path=path, next_norm=(g, EPS))
    ml.check_device_status()
    assert rb0.normed is None and rb1.normed is not None
    assert torch.equal(rb0.indices, rb1.indices)
    assert np.array_equal(bits_of(y0), bits_of(y1))
    _check_norm(bits_of(rb1.normed), orc.rms_norm_bits(bits_of(y1), bits_of(g), EPS))


def test_ep_combine_next_norm():
    """The expert-parallel backend's combine with the fused norm (returned rows already local)."""
    from kcapw_klcquant_b200.ep import CudaBackend

    rng = np.random.default_rng(11)
    T, k, H = 8, 4, 256
    y_bits = _bf16_bits(rng.standard_normal((T * k, H)))
    pair_pos = rng.permutation(T * k).astype(np.int32)
    w_bits = _bf16_bits(rng.random((T, k)) / k)
    res_bits = _bf16_bits(rng.standard_normal((T, H)))
    g_bits = _bf16_bits(1.0 + 0.1 * rng.standard_normal(H))
    backend = CudaBackend.__new__(CudaBackend)  # combine needs only the device
    backend.device = DEV
    y, pp, w, g, res = _dev(y_bits), torch.from_numpy(pair_pos).to(DEV), _dev(w_bits), _dev(g_bits), _dev(res_bits)
    out, normed = backend.combine(y, pp, w, residual=res, next_norm=(g, EPS))
    plain = backend.combine(y, pp, w, residual=res)
    want = _residual_add_bits(orc.combine_bits(orc.bf16_bits_to_f32(y_bits)[pair_pos].reshape(T, k, H), w_bits), res_bits)
    assert np.array_equal(bits_of(out), want) and np.array_equal(bits_of(plain), want)
    _check_norm(bits_of(normed), orc.rms_norm_bits(want, g_bits, EPS))


@pytest.mark.parametrize("T,k,H,E,kn", [(1, 4, 2880, 128, 4), (7, 4, 2880, 128, 4), (64, 4, 2880, 32, 2), (100, 4, 2880, 128, 4),
                                        (5, 2, 256, 200, 8)])
def test_combine_rmsnorm_next_router_vs_oracle(T, k, H, E, kn):
    """klc_moe_combine_rmsnorm_route: the same residual sum and norm as
    klc_moe_combine_rmsnorm, and the next layer's routing of the normalised rows
    held to the router's bar (logits within 1 ulp or the fp32 summation bound of
    the oracle's, a valid top-k of them, weights the softmax of the selected)."""
    from kcapw_klcquant_b200 import _lib

    rng = np.random.default_rng(T * 17 + E)
    R = T * k + 3
    y_bits = _bf16_bits(rng.standard_normal((R, H)) * 2.0)
    pair_pos = rng.permutation(R)[: T * k].astype(np.int32)
    w_bits = _bf16_bits(rng.random((T, k)) / k)
    res_bits = _bf16_bits(rng.standard_normal((T, H)) * 4.0)
    g_bits = _bf16_bits(1.0 + 0.1 * rng.standard_normal(H))
    rw_bits = _bf16_bits(rng.standard_normal((E, H)) * 0.05)
    rb_bits = _bf16_bits(rng.standard_normal(E) * 0.1)
    y, pp, w, g, res = _dev(y_bits), torch.from_numpy(pair_pos).to(DEV), _dev(w_bits), _dev(g_bits), _dev(res_bits)
    rw, rb = _dev(rw_bits), _dev(rb_bits)
    out, normed = torch.empty((T, H), dtype=torch.bfloat16, device=DEV), torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
    out0, normed0 = torch.empty_like(out), torch.empty_like(out)
    nidx = torch.empty((T, kn), dtype=torch.int32, device=DEV)
    nw = torch.empty((T, kn), dtype=torch.bfloat16, device=DEV)
    nlg = torch.empty((T, E), dtype=torch.bfloat16, device=DEV)
    nr = _lib.KlcNextRouter(rw.data_ptr(), rb.data_ptr(), E, kn, nidx.data_ptr(), nw.data_ptr(), nlg.data_ptr())
    L = _lib.lib()
    with torch.cuda.device(DEV):
        _lib.check(L.klc_moe_combine_rmsnorm_route(y.data_ptr(), pp.data_ptr(), w.data_ptr(), T, k, H, res.data_ptr(), g.data_ptr(),
                                                   EPS, out.data_ptr(), normed.data_ptr(), nr, _lib.stream_ptr()))
        _lib.check(L.klc_moe_combine_rmsnorm(y.data_ptr(), pp.data_ptr(), w.data_ptr(), T, k, H, res.data_ptr(), g.data_ptr(), EPS,
                                             out0.data_ptr(), normed0.data_ptr(), _lib.stream_ptr()))
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(out), bits_of(out0))
    assert np.array_equal(bits_of(normed), bits_of(normed0))
    n_bits = bits_of(normed)
    ref = orc.router_logits_bits(n_bits, rw_bits, rb_bits)
    got = bits_of(nlg)
    d = parity.ulp_distance_bf16(got, ref)
    xf, wf = orc.bf16_bits_to_f32(n_bits).astype(np.float64), orc.bf16_bits_to_f32(rw_bits).astype(np.float64)
    mag = np.abs(xf) @ np.abs(wf).T + np.abs(orc.bf16_bits_to_f32(rb_bits))
    err = np.abs(orc.bf16_bits_to_f32(got).astype(np.float64) - orc.bf16_bits_to_f32(ref))
    assert ((d <= 1) | (err <= mag * 2.0**-18)).all(), int(d.max())
    got_idx = nidx.cpu().numpy()
    parity.check_selection(got, got_idx, kn)
    scores = np.take_along_axis(orc.bf16_bits_to_f32(got), got_idx.astype(np.int64), axis=1)
    wd = parity.ulp_distance_bf16(bits_of(nw), orc.softmax_weights_bits(scores))
    assert wd.max() <= 1


def test_stack_fused_router_matches_unfused():
    """A 3-layer MoeStack with each layer's router fused into the previous combine
    against the same stack routing every layer itself: same routing (up to exact
    near-ties of the two router forms) and outputs."""
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200.stack import MoeStack
    from kcapw_klcquant_b200 import synthetic as syn

    dims = syn.LayerDims(32, 2880, 2880, 4)
    layers = [MoeLayer.from_tensors(0, syn.make_layer(dims, seed=90 + i, device=DEV), DEV, top_k=4) for i in range(3)]
    norms = [syn.make_rms_weight(2880, seed=95 + i, device=DEV) for i in range(3)]
    x = syn.make_hidden(24, 2880, seed=99, device=DEV)
    fused = MoeStack(layers, norms, fuse_router=True).step(x)
    plain = MoeStack(layers, norms, fuse_router=False).step(x)
    torch.cuda.synchronize()
    m = parity.assert_output_close(bits_of(fused), bits_of(plain), "stack fused router vs plain")
    assert m["bit_equal_frac"] >= 0.99, m
