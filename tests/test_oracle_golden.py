"""Pin the CPU oracle against fixtures produced by the reference itself.

The fixtures in tests/golden/ were written by tests/golden/make_golden.py,
which runs the reference's own functions; these tests check that the numpy
restatement in oracle/moe_oracle.py reproduces them.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import moe_oracle as orc
from tests import parity
from tests.golden import cases

SMALL_CASES = cases.SMALL_LAYOUT_CASES
BIG_CASES = cases.FULL_LAYOUT_CASES


def _fixture_exists(name):
    return (cases.HERE / f"route_{name}.npz").exists()


# ---------------------------------------------------------------------------
# dequant: bit-exact over all 256 scales x 16 nibbles, three dtypes
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("tag", ["table", "rand"])
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_dequant_bits(golden_dir, tag, dtype):
    fx = np.load(golden_dir / "dequant.npz")
    got = orc.dequantize_mxfp4_bits(fx[f"{tag}_blocks"], fx[f"{tag}_scales"], dtype)
    np.testing.assert_array_equal(got, fx[f"{tag}_{dtype}"])


def test_dequant_shape_mismatch_raises():
    with pytest.raises(ValueError):
        orc.dequantize_mxfp4_exact(np.zeros((4, 2, 16), np.uint8), np.zeros((4, 3), np.uint8))


# ---------------------------------------------------------------------------
# router: logits (ulp-level), tie-aware selection, softmax weights (bit-exact)
# ---------------------------------------------------------------------------


def _route_case(name):
    if not _fixture_exists(name):
        pytest.skip(f"fixture route_{name}.npz not generated")
    return cases.load_route_case(name)


@pytest.mark.parametrize("name", SMALL_CASES)
def test_router_logits(name):
    fx, dims, layer, x = _route_case(name)
    got = orc.router_logits_bits(cases.bits(x), cases.bits(layer["model.layers.0.mlp.router.weight"]), cases.bits(layer["model.layers.0.mlp.router.bias"]))
    d = parity.ulp_distance_bf16(got, fx["logits"])
    assert d.max() <= 1, d.max()
    assert np.mean(d > 0) <= 0.01


@pytest.mark.parametrize("name", SMALL_CASES)
def test_router_selection_and_weights(name):
    fx, dims, layer, x = _route_case(name)
    k = dims.top_k
    lg = orc.bf16_bits_to_f32(fx["logits"])
    idx, scores = orc.select_topk(lg, k)
    parity.check_selection(fx["logits"], idx, k)
    for precision in ("fp32", "bf16"):
        ref_idx = fx[f"experts_{precision}"]
        parity.check_selection(fx["logits"], ref_idx, k, strict_tie_order=False) if name.startswith("tie") else np.testing.assert_array_equal(idx, ref_idx)
        parity.same_selection_modulo_ties(fx["logits"], ref_idx, idx, k)
        # weights are softmax over the reference's own selected scores
        ref_scores = np.take_along_axis(lg, ref_idx.astype(np.int64), axis=1)
        w = orc.softmax_weights_bits(ref_scores)
        np.testing.assert_array_equal(w, fx[f"weights_{precision}"])


def test_tie_case_has_ties():
    fx, dims, layer, x = _route_case("tie_e16_h64_t24")
    ties = parity.check_selection(fx["logits"], fx["experts_fp32"], dims.top_k, strict_tie_order=False)
    assert ties > 0


# ---------------------------------------------------------------------------
# experts + combine, replaying the reference's routing
# ---------------------------------------------------------------------------


def _replay(fx, dims, layer, x, precision, intermediates=False):
    p = "model.layers.0.mlp"
    ex = orc.DenseExperts(
        cases.bits(layer[f"{p}.experts.gate_up_proj_blocks"]),
        cases.bits(layer[f"{p}.experts.gate_up_proj_scales"]),
        cases.bits(layer[f"{p}.experts.down_proj_blocks"]),
        cases.bits(layer[f"{p}.experts.down_proj_scales"]),
    )
    return orc.moe_layer(
        cases.bits(x),
        fx[f"experts_{precision}"],
        fx[f"weights_{precision}"],
        ex,
        cases.bits(layer[f"{p}.experts.gate_up_proj_bias"]),
        cases.bits(layer[f"{p}.experts.down_proj_bias"]),
        precision,
        return_intermediates=intermediates,
    )


@pytest.mark.parametrize("name", SMALL_CASES)
@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_moe_outputs(name, precision):
    fx, dims, layer, x = _route_case(name)
    y, inter = _replay(fx, dims, layer, x, precision, intermediates=True)
    m = parity.assert_output_close(y, fx[f"out_{precision}"], f"{name}/{precision}")
    # the restatement is within a couple of bf16 ulps of the reference
    assert parity.ulp_distance_bf16(y, fx[f"out_{precision}"]).max() <= 4, m
    if f"gu_{precision}" in fx:
        nt = fx[f"gu_{precision}"].shape[0]
        np.testing.assert_allclose(inter["gu"][:nt], fx[f"gu_{precision}"], rtol=2e-5, atol=2e-4)
        np.testing.assert_allclose(inter["gated"][:nt], fx[f"gated_{precision}"], rtol=2e-5, atol=2e-4)
    # expert_logs norms (streamed_moe_router.py:514-521)
    norms = np.stack([np.linalg.norm(inter["gated"].astype(np.float64), axis=-1), np.linalg.norm(inter["out"].astype(np.float64), axis=-1)], -1)
    np.testing.assert_allclose(norms, fx[f"norms_{precision}"], rtol=1e-4)


@pytest.mark.parametrize("name", SMALL_CASES)
def test_bias_only_path(name):
    fx, dims, layer, x = _route_case(name)
    y = orc.bias_only_bits(fx["experts_fp32"], fx["weights_fp32"], cases.bits(layer["model.layers.0.mlp.experts.down_proj_bias"]))
    assert parity.ulp_distance_bf16(y, fx["out_bias_only"]).max() <= 1


@pytest.mark.slow
@pytest.mark.parametrize("name", BIG_CASES)
def test_full_size_layer(name):
    """Full layouts (H = I = 2880): routing exact modulo ties, outputs within tolerance."""
    fx, dims, layer, x = _route_case(name)
    lg = orc.bf16_bits_to_f32(fx["logits"])
    idx, _ = orc.select_topk(lg, dims.top_k)
    parity.same_selection_modulo_ties(fx["logits"], fx["experts_fp32"], idx, dims.top_k)
    got_logits = orc.router_logits_bits(cases.bits(x), cases.bits(layer["model.layers.0.mlp.router.weight"]), cases.bits(layer["model.layers.0.mlp.router.bias"]))
    assert parity.ulp_distance_bf16(got_logits, fx["logits"]).max() <= 1
    # replay the first tokens only (each touches up to k experts of 25 M weights)
    nt = 3
    sub = dict(fx)
    for precision in ("fp32", "bf16"):
        sub[f"experts_{precision}"] = fx[f"experts_{precision}"][:nt]
        sub[f"weights_{precision}"] = fx[f"weights_{precision}"][:nt]
        y = _replay(sub, dims, layer, x[:nt], precision)
        parity.assert_output_close(y, fx[f"out_{precision}"][:nt], f"{name}/{precision}")


# ---------------------------------------------------------------------------
# permutation restatement
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("pad", [1, 8, 16])
def test_permute_is_stable_grouping(pad):
    rng = np.random.default_rng(3)
    E, T, k = 12, 50, 3
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
    rows, counts, offsets = orc.moe_permute(idx, E, pad)
    flat = idx.reshape(-1)
    assert counts.sum() == T * k
    for e in range(E):
        seg = rows[offsets[e] : offsets[e] + counts[e]]
        assert np.all(flat[seg] == e)
        assert np.all(np.diff(seg) > 0)
        assert np.all(rows[offsets[e] + counts[e] : offsets[e + 1]] == -1)
        assert (offsets[e + 1] - offsets[e]) % pad == 0


# ---------------------------------------------------------------------------
# rms_norm and the runtime dequantizer
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("H", [2880, 128])
def test_rms_norm(golden_dir, H):
    fx = np.load(golden_dir / "rmsnorm.npz")
    y = orc.rms_norm_bits(fx[f"h{H}_x"], fx[f"h{H}_w"], 1e-5)
    d = parity.ulp_distance_bf16(y, fx[f"h{H}_y"])
    assert d.max() <= 1 and np.mean(d > 0) < 0.01


@pytest.mark.parametrize("mode", ["q1", "q2", "q3", "q4", "q8", "q16", "fp16"])
@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_runtime_dequant(golden_dir, mode, dtype):
    fx = np.load(golden_dir / "runtime_dequant.npz")
    shape = tuple(int(v) for v in fx["shape"])
    bits, packed = (int(v) for v in fx[f"{mode}_meta"])
    data = fx[f"{mode}_data"]
    if str(fx[f"{mode}_data_dtype"]) == "torch.float16":
        data = data.view(np.float16)
    got = orc.runtime_dequantize_bits(mode, data, fx[f"{mode}_scale"], shape, dtype, bits, bool(packed))
    np.testing.assert_array_equal(got, fx[f"{mode}_{dtype}"])


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_runtime_dequant_pruned(golden_dir, dtype):
    fx = np.load(golden_dir / "runtime_dequant.npz")
    shape = tuple(int(v) for v in fx["shape"])
    got = orc.reconstruct_pruned_bits(orc.bf16_bits_to_f32(fx["pruned_values"]), fx["pruned_indices"], shape, dtype)
    np.testing.assert_array_equal(got, fx[f"pruned_{dtype}"])
