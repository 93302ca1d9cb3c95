"""GPU parity of the CUDA path against the reference fixtures and the CPU oracle.

Every compute call goes through the C ABI of libklcmoe.so (via the
package's thin ctypes wrappers).  Bit-exact where the reference is exact
(dequant, routing indices modulo exact ties, permutation, combine); within
the stated tolerance for the floating-point expert GEMMs:
cosine >= 0.9999 and max-abs / max|ref| <= 2e-2.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests import parity
from tests.golden import cases

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
SMALL_CASES = cases.SMALL_LAYOUT_CASES
ALL_CASES = list(cases.ROUTE_CASES)


def _paths():
    from kcapw_klcquant_b200 import _lib

    return sorted(_lib.capabilities())


PATHS = _paths() if torch.cuda.is_available() else ["simt"]


@pytest.fixture(scope="module")
def case_cache():
    return {}


def load(case_cache, name):
    if name not in case_cache:
        fx, dims, layer, x = cases.load_route_case(name)
        from kcapw_klcquant_b200 import MoeLayer

        ml = MoeLayer.from_tensors(0, layer, DEV, top_k=dims.top_k)
        case_cache[name] = (fx, dims, layer, x, ml)
    return case_cache[name]


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------------------
# dequant
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("tag", ["table", "rand"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_dequant_golden(golden_dir, tag, dtype):
    from kcapw_klcquant_b200 import dequantize_mxfp4_matrix

    fx = np.load(golden_dir / "dequant.npz")
    b = torch.from_numpy(fx[f"{tag}_blocks"]).to(DEV)
    s = torch.from_numpy(fx[f"{tag}_scales"]).to(DEV)
    out = dequantize_mxfp4_matrix(b, s, dtype).cpu()
    key = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    got = out.view(torch.int32).numpy().view(np.uint32) if dtype == torch.float32 else out.view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, fx[f"{tag}_{key}"])


def test_dequant_full_expert_vs_oracle():
    from kcapw_klcquant_b200 import dequantize_mxfp4_matrix

    g = torch.Generator().manual_seed(9)
    b = torch.randint(0, 256, (5760, 90, 16), generator=g, dtype=torch.uint8)
    s = torch.randint(0, 256, (5760, 90), generator=g, dtype=torch.uint8)
    got = bits_of(dequantize_mxfp4_matrix(b.to(DEV), s.to(DEV), torch.bfloat16))
    ref = orc.dequantize_mxfp4_bits(b.numpy(), s.numpy(), "bf16")
    np.testing.assert_array_equal(got, ref)


def test_dequant_shape_mismatch():
    from kcapw_klcquant_b200 import dequantize_mxfp4_matrix

    with pytest.raises(ValueError):
        dequantize_mxfp4_matrix(torch.zeros(4, 2, 16, dtype=torch.uint8, device=DEV), torch.zeros(4, 3, dtype=torch.uint8, device=DEV))


# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("name", ALL_CASES)
def test_router_vs_reference(case_cache, name):
    fx, dims, layer, x, ml = load(case_cache, name)
    from kcapw_klcquant_b200 import _lib

    T, k, E = x.shape[0], dims.top_k, dims.experts
    xd = x.to(DEV)
    idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=DEV)
    lg = torch.empty((T, E), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().klc_router_topk(xd.data_ptr(), T, dims.hidden, ml.router_weight.data_ptr(), ml.router_bias.data_ptr(), E, k, None,
                                          idx.data_ptr(), w.data_ptr(), lg.data_ptr(), _lib.stream_ptr()))
    got_logits = bits_of(lg)
    d = parity.ulp_distance_bf16(got_logits, fx["logits"])
    assert d.max() <= 1, d.max()
    assert np.mean(d > 0) <= 0.01
    got_idx = idx.cpu().numpy()
    # selection is a valid top-k of our own logits with the lower-index tie rule
    parity.check_selection(got_logits, got_idx, k)
    # and equals the reference's selection wherever the logits agree exactly
    same_rows = np.all(got_logits == fx["logits"], axis=1)
    parity.same_selection_modulo_ties(fx["logits"][same_rows], fx["experts_fp32"][same_rows], got_idx[same_rows], k)
    # weights: softmax of our selected scores, bit-exact vs the oracle
    scores = np.take_along_axis(orc.bf16_bits_to_f32(got_logits), got_idx.astype(np.int64), axis=1)
    wd = parity.ulp_distance_bf16(bits_of(w), orc.softmax_weights_bits(scores))
    assert wd.max() <= 1 and np.mean(wd > 0) <= 0.02
    # rows with identical logits and no tie: weights equal the reference's exactly (up to expf ulps)
    ref_w = fx["weights_fp32"]
    rw = parity.ulp_distance_bf16(bits_of(w)[same_rows], ref_w[same_rows])
    if not name.startswith("tie"):
        assert rw.max() <= 1 and np.mean(rw > 0) <= 0.02


def test_select_softmax_keep_order():
    from kcapw_klcquant_b200 import _lib

    s = torch.tensor([[0.3, 1.2, -0.5, 0.9]], dtype=torch.float32, device=DEV)
    w = torch.empty((1, 4), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().klc_select_softmax(s.data_ptr(), 1, 4, 4, 1, None, w.data_ptr(), _lib.stream_ptr()))
    np.testing.assert_array_equal(bits_of(w)[0], orc.softmax_weights_bits(s.cpu().numpy())[0])


# Every router form against the oracle's logits (fp32 accumulation, one bf16
# rounding): E <= 128 with H a multiple of 64 runs the tensor-core split-K
# router, the other shapes the CUDA-core router; token counts cross the
# 16 / 32 / 64-token tile choices; from 1024 tokens the large-batch router
# (128-token tiles, the hidden dimension split over a cluster of 8 or 4 CTAs
# or whole), also with expert counts below its padded width (32, 48, 100, 200).
@pytest.mark.parametrize("T,E,H,k", [(1, 128, 2880, 4), (37, 32, 2880, 4), (300, 128, 2880, 4), (5000, 128, 2880, 4),
                                     (20, 8, 64, 2), (33, 128, 3072, 4), (40, 192, 256, 4), (24, 64, 200, 3),
                                     (2100, 32, 2880, 4), (2048, 48, 1024, 2), (2300, 200, 512, 8), (1500, 128, 2880, 4),
                                     (1100, 100, 1536, 3)])
def test_router_shapes_vs_oracle(T, E, H, k):
    from kcapw_klcquant_b200 import _lib

    rng = np.random.default_rng(T * 7 + E)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16)
    wr = torch.from_numpy((rng.standard_normal((E, H)) * 0.05).astype(np.float32)).to(torch.bfloat16)
    br = torch.from_numpy((rng.standard_normal(E) * 0.1).astype(np.float32)).to(torch.bfloat16)
    xd, wd, bd = x.to(DEV), wr.to(DEV), br.to(DEV)
    idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=DEV)
    lg = torch.empty((T, E), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().klc_router_topk(xd.data_ptr(), T, H, wd.data_ptr(), bd.data_ptr(), E, k, None, idx.data_ptr(),
                                          w.data_ptr(), lg.data_ptr(), _lib.stream_ptr()))
    assert _lib.lib().klc_router_status(None, None, _lib.stream_ptr()) == _lib.KLC_OK
    ref = orc.router_logits_bits(bits_of(x), bits_of(wr), bits_of(br))
    got = bits_of(lg)
    d = parity.ulp_distance_bf16(got, ref)
    assert np.mean(d > 0) <= 0.01
    # one bf16 ulp, or (near-cancelling sums) an fp32 accumulation error of at most
    # 2^-18 of the sum of |products|: fp32 sums in another order than the oracle's
    xf, wf = x.float().numpy(), wr.float().numpy()
    mag = np.abs(xf) @ np.abs(wf).T + np.abs(br.float().numpy())
    err = np.abs(orc.bf16_bits_to_f32(got).astype(np.float64) - orc.bf16_bits_to_f32(ref))
    ok = (d <= 1) | (err <= mag * 2.0**-18)
    assert ok.all(), (d.max(), float((err / mag).max()))
    got_idx = idx.cpu().numpy()
    parity.check_selection(got, got_idx, k)
    scores = np.take_along_axis(orc.bf16_bits_to_f32(got), got_idx.astype(np.int64), axis=1)
    wdist = parity.ulp_distance_bf16(bits_of(w), orc.softmax_weights_bits(scores))
    assert wdist.max() <= 1 and np.mean(wdist > 0) <= 0.02


@pytest.mark.parametrize("T", [100, 4096])
def test_router_exact_ties_lower_index_first(T):
    """Router rows duplicated in pairs: every token has exact ties at every rank of
    its top-k.  Both router forms (the cluster form at T = 100, the whole-K GEMM
    form at T = 4096) must order equal values by the lower expert index."""
    from kcapw_klcquant_b200 import _lib

    E, H, k = 64, 256, 5
    rng = np.random.default_rng(T)
    half = (rng.standard_normal((E // 2, H)) * 0.05).astype(np.float32)
    wr = torch.from_numpy(np.repeat(half, 2, axis=0)[rng.permutation(E)].copy()).to(torch.bfloat16)
    br = torch.zeros(E, dtype=torch.bfloat16)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16)
    idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=DEV)
    lg = torch.empty((T, E), dtype=torch.bfloat16, device=DEV)
    xd, wd, bd = x.to(DEV), wr.to(DEV), br.to(DEV)
    _lib.check(_lib.lib().klc_router_topk(xd.data_ptr(), T, H, wd.data_ptr(), bd.data_ptr(), E, k, None, idx.data_ptr(),
                                          w.data_ptr(), lg.data_ptr(), _lib.stream_ptr()))
    got = bits_of(lg)
    ties = parity.check_selection(got, idx.cpu().numpy(), k)
    assert ties > 0
    scores = np.take_along_axis(orc.bf16_bits_to_f32(got), idx.cpu().numpy().astype(np.int64), axis=1)
    assert parity.ulp_distance_bf16(bits_of(w), orc.softmax_weights_bits(scores)).max() <= 1


# ---------------------------------------------------------------------------
# permutation (bit-exact vs the stable-sort oracle)
# ---------------------------------------------------------------------------


# up to 16384 pairs the permute is one fused launch, above it three launches
@pytest.mark.parametrize("skew", [False, True])
@pytest.mark.parametrize("T,k,E", [(1, 4, 128), (5, 2, 8), (300, 4, 128), (4096, 4, 128), (4097, 4, 128), (2000, 3, 37),
                                   (9000, 2, 1024)])
def test_permute_exact(T, k, E, skew):
    import ctypes
    from kcapw_klcquant_b200 import _lib

    rng = np.random.default_rng(T + E)
    p = None
    if skew:  # most pairs on a handful of experts (contended histogram bins)
        p = 1.0 / np.arange(1, E + 1) ** 2.0
        p /= p.sum()
    idx = np.stack([rng.choice(E, k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    pad = 16
    rows_cap = T * k + E * (pad - 1)
    d_idx = torch.from_numpy(idx).to(DEV)
    pair_pos = torch.empty(T * k, dtype=torch.int32, device=DEV)
    counts = torch.empty(E, dtype=torch.int32, device=DEV)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=DEV)
    rows = torch.full((rows_cap,), -7, dtype=torch.int32, device=DEV)
    dims = _lib.KlcDims(T, 64, 64, E, k, _lib.KLC_PATH_SIMT)
    n = ctypes.c_size_t(0)
    _lib.check(_lib.lib().klc_moe_workspace_size(ctypes.byref(dims), ctypes.byref(n)))
    ws = torch.empty(n.value, dtype=torch.uint8, device=DEV)
    _lib.check(_lib.lib().klc_moe_permute(d_idx.data_ptr(), T, k, E, pad, pair_pos.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                                          rows.data_ptr(), rows_cap, ws.data_ptr(), ws.numel(), _lib.stream_ptr()))
    r_rows, r_counts, r_off = orc.moe_permute(idx, E, pad)
    np.testing.assert_array_equal(counts.cpu().numpy(), r_counts)
    np.testing.assert_array_equal(offsets.cpu().numpy(), r_off)
    np.testing.assert_array_equal(rows.cpu().numpy()[: r_off[-1]], r_rows)
    pp = pair_pos.cpu().numpy()
    np.testing.assert_array_equal(r_rows[pp], np.arange(T * k))


def test_permute_rejects_bad_expert_index():
    import ctypes
    from kcapw_klcquant_b200 import _lib

    T, k, E = 4, 2, 8
    idx = torch.tensor([[0, 1], [2, 9], [3, 4], [5, 6]], dtype=torch.int32, device=DEV)
    rows_cap = T * k + E * 15
    outs = [torch.empty(n, dtype=torch.int32, device=DEV) for n in (T * k, E, E + 1, rows_cap)]
    dims = _lib.KlcDims(T, 64, 64, E, k, _lib.KLC_PATH_SIMT)
    n = ctypes.c_size_t(0)
    _lib.check(_lib.lib().klc_moe_workspace_size(ctypes.byref(dims), ctypes.byref(n)))
    ws = torch.empty(n.value, dtype=torch.uint8, device=DEV)
    _lib.check(_lib.lib().klc_moe_permute(idx.data_ptr(), T, k, E, 16, *(o.data_ptr() for o in outs), rows_cap, ws.data_ptr(), ws.numel(), _lib.stream_ptr()))
    st = _lib.lib().klc_workspace_status(ws.data_ptr(), None, None, None, _lib.stream_ptr())
    assert st == _lib.KLC_ERR_DEVICE_FAULT


# ---------------------------------------------------------------------------
# experts + combine, replaying the reference's routing
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("precision", ["fp32", "bf16"])
@pytest.mark.parametrize("name", ALL_CASES)
def test_experts_replay_vs_reference(case_cache, name, precision, path):
    fx, dims, layer, x, ml = load(case_cache, name)
    idx = torch.from_numpy(fx[f"experts_{precision}"].astype(np.int32))
    w = torch.from_numpy(fx[f"weights_{precision}"].view(np.int16)).view(torch.bfloat16)
    y, norms = ml.experts_forward(x.to(DEV), idx, w, precision=precision, return_norms=True, path=path)
    ml.check_device_status()
    m = parity.assert_output_close(bits_of(y), fx[f"out_{precision}"], f"{name}/{precision}/{path}")
    if path == "simt":
        # fp32 CUDA-core math: only the summation order differs from the
        # reference, so almost every output is bit-identical
        assert m["bit_equal_frac"] >= 0.99, m
    np.testing.assert_allclose(norms.cpu().numpy(), fx[f"norms_{precision}"], rtol=5e-3 if path == "tc" else 1e-4)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", SMALL_CASES)
def test_forward_end_to_end(case_cache, name, path):
    """Router + experts + combine in one call vs the reference's route() per token."""
    fx, dims, layer, x, ml = load(case_cache, name)
    y, rb = ml.forward(x.to(DEV), precision="bf16", return_logits=True, path=path)
    ml.check_device_status()
    got_logits = bits_of(rb.logits)
    got_idx = rb.indices.cpu().numpy()
    parity.check_selection(got_logits, got_idx, dims.top_k)
    equal_logits = np.all(got_logits == fx["logits"], axis=1)
    parity.same_selection_modulo_ties(fx["logits"][equal_logits], fx["experts_bf16"][equal_logits], got_idx[equal_logits], dims.top_k)
    same = equal_logits & np.all(np.sort(got_idx, 1) == np.sort(fx["experts_bf16"], 1), axis=1)
    if not name.startswith("tie"):  # exact ties may legitimately pick another member of the tied class
        assert same.mean() >= 0.9
    parity.assert_output_close(bits_of(y)[same], fx["out_bf16"][same], f"{name}/{path}")


def test_bias_only(case_cache):
    fx, dims, layer, x, ml = load(case_cache, "mini_e16_h256_t32")
    from kcapw_klcquant_b200 import _lib

    T, k = x.shape[0], dims.top_k
    idx = torch.from_numpy(fx["experts_fp32"].astype(np.int32)).to(DEV)
    w = torch.from_numpy(fx["weights_fp32"].view(np.int16)).view(torch.bfloat16).to(DEV)
    y = torch.empty((T, dims.hidden), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().klc_moe_bias_only(ml.down_bias.data_ptr(), T, dims.hidden, k, idx.data_ptr(), w.data_ptr(), y.data_ptr(), _lib.stream_ptr()))
    assert parity.ulp_distance_bf16(bits_of(y), fx["out_bias_only"]).max() <= 1


# ---------------------------------------------------------------------------
# drop-in API: StreamedMoERouter.route / route_batch, Mxfp4ExpertStore
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_route_dropin(case_cache, precision):
    from kcapw_klcquant_b200 import Mxfp4ExpertStore, StreamedMoERouter
    from kcapw_klcquant_b200 import synthetic as syn

    fx, dims, layer, x, ml = load(case_cache, "mini_e8_h128_i192_t6")
    store = Mxfp4ExpertStore.from_layers({0: layer}, DEV)
    router = StreamedMoERouter(experts_per_token=dims.top_k, swiglu_limit=7.0, matmul_precision=precision)
    tensors = {k: v.to(DEV) for k, v in syn.dense_tensors(layer).items()}
    for t in range(x.shape[0]):
        y, route = router.route(0, x[t].to(DEV), tensors, store, True, t)
        assert route["mode"] == "mxfp4_expert_matmul"
        assert set(route) >= {"experts", "weights", "expert_logs", "raw_experts", "predicted_experts", "resident_experts", "sticky_adjusted", "active_expert_cap"}
        assert route["experts"] == [int(v) for v in fx[f"experts_{precision}"][t]]
        parity.assert_output_close(bits_of(y.reshape(1, -1)), fx[f"out_{precision}"][t : t + 1], f"route t={t}")
    js = router.stats.to_json()
    assert js["routed_tokens"] == x.shape[0]
    # bias-only mode
    y, route = router.route(0, x[0].to(DEV), tensors, None, False, 0)
    assert route["mode"] == "bias_only_moe"
    assert parity.ulp_distance_bf16(bits_of(y.reshape(1, -1)), fx["out_bias_only"][:1]).max() <= 1


def test_route_batch_matches_route_and_records_stats(case_cache):
    """route_batch() over T tokens equals route() per token (locality off), and its
    statistics, copied asynchronously, appear in order once the stats are read."""
    from kcapw_klcquant_b200 import Mxfp4ExpertStore, StreamedMoERouter
    from kcapw_klcquant_b200 import synthetic as syn

    fx, dims, layer, x, ml = load(case_cache, "mini_e16_h256_t32")
    store = Mxfp4ExpertStore.from_layers({0: layer}, DEV)
    tensors = {k: v.to(DEV) for k, v in syn.dense_tensors(layer).items()}
    rb_router = StreamedMoERouter(dims.top_k, 7.0, matmul_precision="bf16")
    y, rb = rb_router.route_batch(0, x.to(DEV), tensors, store, record_stats=True, position=10)
    y2, rb2 = rb_router.route_batch(0, x[:5].to(DEV), tensors, store, record_stats=True, position=100)
    assert len(rb_router._pending) == 2  # nothing recorded (no host synchronisation) until the stats are read
    js = rb_router.stats.to_json()
    assert js["routed_tokens"] == x.shape[0] + 5 and not rb_router._pending
    ev = js["route_events"]
    assert [e["position"] for e in ev] == list(range(10, 10 + x.shape[0])) + list(range(100, 105))
    assert [e["experts"] for e in ev[: x.shape[0]]] == rb.indices.tolist()
    per_token = StreamedMoERouter(dims.top_k, 7.0, matmul_precision="bf16")
    for t in range(x.shape[0]):
        yt, route = per_token.route(0, x[t].to(DEV), tensors, store, True, t)
        assert route["experts"] == rb.indices[t].tolist()
        assert torch.equal(yt.reshape(-1), y[t])


def test_store_load_expert_matrix_matches_dequant(case_cache):
    from kcapw_klcquant_b200 import Mxfp4ExpertStore

    fx, dims, layer, x, ml = load(case_cache, "mini_e16_h256_t32")
    store = Mxfp4ExpertStore.from_layers({0: layer}, DEV, dtype=torch.bfloat16, cache_bytes=1 << 30)
    m = store.load_expert_matrix(0, 3, "gate_up_proj")
    ref = orc.dequantize_mxfp4_bits(cases.bits(layer["model.layers.0.mlp.experts.gate_up_proj_blocks"][3]),
                                    cases.bits(layer["model.layers.0.mlp.experts.gate_up_proj_scales"][3]), "bf16")
    np.testing.assert_array_equal(bits_of(m), ref)
    store.load_expert_matrix(0, 3, "gate_up_proj")
    assert store.cache.stats.hits == 1 and store.cache.stats.misses == 1
    assert store.resident_experts(0) == set(range(dims.experts))


@pytest.mark.parametrize("name", list(cases.LOCALITY_CASES))
def test_locality_route_vs_reference(golden_dir, name):
    """route() with the locality policy on the device path against the reference's
    route() on the same token sequence: routing dicts, outputs and to_json()."""
    import json

    from kcapw_klcquant_b200 import Mxfp4ExpertStore, RoutingLocalityConfig, StreamedMoERouter
    from kcapw_klcquant_b200 import synthetic as syn

    E, H, I, k, T, seed, execute, cfg_kw = cases.LOCALITY_CASES[name]
    fx = np.load(golden_dir / f"locality_{name}.npz")
    ref_routes = json.loads(str(fx["routes_json"]))
    layer = syn.make_layer(syn.LayerDims(E, H, I, k), seed)
    x = cases.correlated_hidden(T, H, seed).to(DEV)
    store = Mxfp4ExpertStore.from_layers({0: layer}, DEV, cache_bytes=1 << 40) if execute else None
    cfg = RoutingLocalityConfig(**cfg_kw) if cfg_kw is not None else None
    router = StreamedMoERouter(k, 7.0, cfg, matmul_precision="bf16")
    tensors = {kk: v.to(DEV) for kk, v in syn.dense_tensors(layer).items()}
    w_r, b_r = tensors["model.layers.0.mlp.router.weight"], tensors["model.layers.0.mlp.router.bias"]
    from kcapw_klcquant_b200 import _lib

    prev: list[int] = []
    for t in range(T):
        # the device logits of this token; the comparison holds while they equal the reference's
        lg = torch.empty((1, E), dtype=torch.bfloat16, device=DEV)
        idx = torch.empty((1, k), dtype=torch.int32, device=DEV)
        w = torch.empty((1, k), dtype=torch.bfloat16, device=DEV)
        _lib.check(_lib.lib().klc_router_topk(x[t : t + 1].contiguous().data_ptr(), 1, H, w_r.data_ptr(), b_r.data_ptr(), E, k, None,
                                              idx.data_ptr(), w.data_ptr(), lg.data_ptr(), _lib.stream_ptr()))
        if not np.array_equal(bits_of(lg)[0], fx["logits"][t]):
            assert parity.ulp_distance_bf16(bits_of(lg)[0], fx["logits"][t]).max() <= 1
            assert t >= T // 2, f"device logits left the reference's at token {t}"
            return
        resident = cases.resident_set(t, prev) if cfg is not None else None
        y, route = router.route(0, x[t], tensors, store, execute, t, resident_experts=resident)
        ref = ref_routes[t]
        for key in ("experts", "raw_experts", "weights", "sticky_adjusted", "mode"):
            assert route.get(key) == ref[key], (t, key, route.get(key), ref[key])
        if execute:
            assert route["predicted_experts"] == ref["predicted_experts"] and route["active_expert_cap"] == ref["active_expert_cap"]
        parity.assert_output_close(bits_of(y.reshape(1, -1)), fx["out"][t : t + 1], f"{name} t={t}")
        prev = [int(e) for e in route["experts"]]
    ref_stats = json.loads(str(fx["stats_json"]))
    got = json.loads(json.dumps(router.stats.to_json()))
    assert got["routed_tokens"] == ref_stats["routed_tokens"]
    assert got["locality"]["dynamic_cap_events"] == ref_stats["locality"]["dynamic_cap_events"]
    assert got["route_events"] == ref_stats["route_events"]
    assert got["cache_delta_events"] == ref_stats["cache_delta_events"]


# ---------------------------------------------------------------------------
# rms_norm, runtime dequantizer
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("H", [2880, 128])
def test_rms_norm(golden_dir, H):
    from kcapw_klcquant_b200 import rms_norm

    fx = np.load(golden_dir / "rmsnorm.npz")
    x = torch.from_numpy(fx[f"h{H}_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    w = torch.from_numpy(fx[f"h{H}_w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    d = parity.ulp_distance_bf16(bits_of(rms_norm(x, w, 1e-5)), fx[f"h{H}_y"])
    assert d.max() <= 1 and np.mean(d > 0) < 0.01


@pytest.mark.parametrize("mode", ["q1", "q2", "q3", "q4", "q8", "q16", "fp16", "pruned"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_runtime_dequantizer(golden_dir, mode, dtype):
    from kcapw_klcquant_b200 import QuantizedTensorMeta, RuntimeDequantizer

    fx = np.load(golden_dir / "runtime_dequant.npz")
    shape = tuple(int(v) for v in fx["shape"])
    key = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    if mode == "pruned":
        meta = QuantizedTensorMeta("t", "pruned", shape, "torch.bfloat16", 16, False, "g", "f")
        data = torch.from_numpy(fx["pruned_values"].view(np.int16)).view(torch.bfloat16)
        scale = torch.from_numpy(fx["pruned_indices"])
    else:
        bits, packed = (int(v) for v in fx[f"{mode}_meta"])
        meta = QuantizedTensorMeta("t", mode, shape, "torch.bfloat16", bits, bool(packed), "g", "f")
        raw = fx[f"{mode}_data"]
        data = torch.from_numpy(raw.view(np.int16)).view(torch.float16) if str(fx[f"{mode}_data_dtype"]) == "torch.float16" else torch.from_numpy(raw)
        scale = torch.from_numpy(fx[f"{mode}_scale"]) if fx[f"{mode}_scale"].size else None
    out = RuntimeDequantizer().dequantize(meta, data, scale, DEV, dtype).cpu()
    got = out.view(torch.int32).numpy().view(np.uint32) if dtype == torch.float32 else out.view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, fx[f"{mode}_{key}"])


def test_runtime_dequantizer_errors():
    from kcapw_klcquant_b200 import QuantizedTensorMeta, RuntimeDequantizer

    meta = QuantizedTensorMeta("t", "q4", (4,), "torch.bfloat16", 4, True, "g", "f")
    with pytest.raises(ValueError):
        RuntimeDequantizer().dequantize(meta, torch.zeros(2, dtype=torch.uint8), None, DEV)
    meta = QuantizedTensorMeta("t", "pruned", (4,), "torch.bfloat16", 16, False, "g", "f")
    with pytest.raises(ValueError):
        RuntimeDequantizer().dequantize(meta, torch.zeros(2, dtype=torch.bfloat16), None, DEV)


# ---------------------------------------------------------------------------
# full-size properties (config-1/2 layouts): determinism, path agreement
# ---------------------------------------------------------------------------


@pytest.fixture(scope="module")
def big_layer():
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn

    dims = syn.GPT_OSS_120B
    layer = syn.make_layer(dims, seed=1, device=DEV)
    return MoeLayer.from_tensors(0, layer, DEV, top_k=4)


# Tile-level races show up as whole tokens that disagree between runs or with
# the CUDA-core path (a wrong 128 x 16 tile of one GEMM perturbs every output
# of its rows), not as a small change of the global tolerance metrics.
@pytest.mark.parametrize("T", [256, 4096])
def test_tensor_core_path_repeatable_per_token(big_layer, T):
    from kcapw_klcquant_b200 import synthetic as syn

    if "tc" not in PATHS:
        pytest.skip("tensor-core path not available")
    x = syn.make_hidden(T, 2880, seed=T + 11, device=DEV)
    ys, _ = big_layer.forward(x, precision="bf16", path="simt")
    runs = []
    for _ in range(3):
        yt, _ = big_layer.forward(x, precision="bf16", path="tc")
        big_layer.check_device_status()
        runs.append(yt.clone())
    for r in runs[1:]:
        assert torch.equal(r, runs[0]), "tensor-core path is not bit-repeatable"
    per_token = (runs[0].view(torch.int16) == ys.view(torch.int16)).float().mean(1)
    assert float(per_token.min()) >= 0.9, (T, int((per_token < 0.9).sum()), float(per_token.min()))


@pytest.mark.parametrize("T", [1, 8, 64, 256, 4096])
def test_full_size_determinism_and_paths(big_layer, T):
    from kcapw_klcquant_b200 import synthetic as syn

    x = syn.make_hidden(T, 2880, seed=T, device=DEV)
    y1, rb1 = big_layer.forward(x, precision="bf16", path="simt")
    y2, rb2 = big_layer.forward(x, precision="bf16", path="simt")
    big_layer.check_device_status()
    assert torch.equal(y1, y2) and torch.equal(rb1.indices, rb2.indices)
    assert torch.isfinite(y1.float()).all()
    counts = torch.bincount(rb1.indices.flatten().long(), minlength=128)
    assert int(counts.sum()) == T * 4
    if "tc" in PATHS:
        y3, rb3 = big_layer.forward(x, precision="bf16", path="tc")
        big_layer.check_device_status()
        assert torch.equal(rb3.indices, rb1.indices)
        parity.assert_output_close(bits_of(y3), bits_of(y1), f"tc vs simt T={T}")


# ---------------------------------------------------------------------------
# the benchmark configurations themselves against the oracle (token subsample)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("T,zipf,seed", [(256, None, 1), (4096, 1.1, 2)])
def test_bench_configs_subsample_vs_oracle(T, zipf, seed, path):
    """Config 1 (decode T=256, uniform) and config 2 (prefill T=4096, Zipf(1.1)
    router) on the full 120B layout: every 4th / 64th token of the batch against
    the oracle on the device's own routing.  At these sizes the tensor-core path
    runs its 16-row (T=256) and 64-row (T=4096, skewed groups) tiles."""
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn

    layer = syn.make_layer(syn.GPT_OSS_120B, seed=seed, zipf=zipf, device=DEV)
    ml = MoeLayer.from_tensors(0, layer, DEV, top_k=4)
    x = syn.make_hidden(T, 2880, seed=seed, device=DEV)
    y, rb = ml.forward(x, precision="bf16", path=path)
    ml.check_device_status()
    counts = torch.bincount(rb.indices.flatten().long(), minlength=128)
    if zipf is not None:
        assert int(counts.max()) > 3 * float(counts.float().mean())  # skewed, load-imbalanced groups
    sample = torch.arange(0, T, T // 64, device=DEV)
    sel = rb.indices[sample].cpu().numpy()
    used = np.unique(sel)
    p = "model.layers.0.mlp.experts"
    host = {n: layer[f"{p}.{n}"][torch.from_numpy(used).to(DEV).long()].cpu().numpy()
            for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")}
    ex = orc.DenseExperts(host["gate_up_proj_blocks"], host["gate_up_proj_scales"], host["down_proj_blocks"], host["down_proj_scales"],
                          max_cached=1)
    remap = np.zeros(128, np.int64)
    remap[used] = np.arange(used.size)
    want = orc.moe_layer(bits_of(x[sample]), remap[sel], bits_of(rb.weights[sample]), ex,
                         bits_of(layer[f"{p}.gate_up_proj_bias"])[used], bits_of(layer[f"{p}.down_proj_bias"])[used], "bf16")
    m = parity.assert_output_close(bits_of(y[sample]), want, f"T={T} zipf={zipf} {path}")
    if path == "simt":
        assert m["bit_equal_frac"] >= 0.99, m


@pytest.mark.parametrize("kernel", ["weights_as_n192", "direct_operand", "repack"])
@pytest.mark.parametrize("name", ["c1_e128_h2880_t8", "mid_zipf_e16_h2880_t64"])
def test_tensor_core_kernel_forms_vs_reference(case_cache, name, kernel):
    """Each tensor-core kernel form against the reference's outputs (replayed routing):
    weights as N = 192 (the default), weights as A with TMA-unpacked operands (no
    192-row scale tiles), and the repack form (no K-padded blocks either).  The
    mid case runs the 64-row tiles, the c1 case the 16-row tiles."""
    import dataclasses

    from kcapw_klcquant_b200 import MoeLayer

    if "tc" not in PATHS:
        pytest.skip("tensor-core path not available")
    fx, dims, layer, x, ml = load(case_cache, name)
    packed = ml.packed
    if kernel != "weights_as_n192":
        packed = dataclasses.replace(packed, gu_scales_t192=None, dn_scales_t192=None)
    if kernel == "repack":
        packed = dataclasses.replace(packed, gu_blocks_k128=None, dn_blocks_k128=None)
    m = MoeLayer(packed, ml.router_weight, ml.router_bias, ml.gate_up_bias, ml.down_bias, top_k=dims.top_k, path="tc")
    for precision in ("bf16", "fp32"):
        idx = torch.from_numpy(fx[f"experts_{precision}"].astype(np.int32))
        w = torch.from_numpy(fx[f"weights_{precision}"].view(np.int16)).view(torch.bfloat16)
        y, norms = m.experts_forward(x.to(DEV), idx, w, precision=precision, return_norms=True)
        m.check_device_status()
        parity.assert_output_close(bits_of(y), fx[f"out_{precision}"], f"{name}/{kernel}/{precision}")
        np.testing.assert_allclose(norms.cpu().numpy(), fx[f"norms_{precision}"], rtol=5e-3)
