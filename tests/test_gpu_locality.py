"""The locality policy on the device (klc_locality_route) against the reference.

1. The reference-generated locality fixtures (tests/golden/locality_*.npz):
   the reference's logits go through the device kernel one token at a time
   (the host applies the dynamic active-expert cap between tokens, as route()
   does), and every per-token decision — raw and guarded experts, weights,
   predictions, the sticky-adjusted flag — and the final RouterStats JSON and
   caps must equal the reference's.
2. Tie-heavy random logits (few distinct values, so exact ties are the rule)
   through one batched call against the host policy (torch.topk on the CPU,
   Python dicts) token by token: same decisions and the same final state.
3. route() and route_batch() with the device policy on real router logits.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.golden import cases
from tests.test_locality_golden import _close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("name", [n for n, spec in cases.LOCALITY_CASES.items() if spec[7] is not None])
def test_device_policy_matches_reference_fixture(golden_dir, name):
    from kcapw_klcquant_b200 import RoutingLocalityConfig, StreamedMoERouter
    from kcapw_klcquant_b200.mxfp4_expert import DenseMatrixCache, account_expert_use

    E, H, I, k_top, T, seed, execute, cfg_kw = cases.LOCALITY_CASES[name]
    fx = np.load(golden_dir / f"locality_{name}.npz")
    ref_routes = json.loads(str(fx["routes_json"]))
    ref_stats = json.loads(str(fx["stats_json"]))
    router = StreamedMoERouter(k_top, 7.0, RoutingLocalityConfig(**cfg_kw), matmul_precision="bf16")
    assert router.locality_on_device
    cache = DenseMatrixCache(1 << 40)
    logits = _bf16(fx["logits"]).to(DEV)
    prev: list[int] = []
    for t in range(T):
        ref = ref_routes[t]
        k = router._effective_expert_count(0, E)
        resident = cases.resident_set(t, prev)
        pol = router._device_policy(0, logits[t:t + 1], k, router._resident_mask(resident, E, DEV), 0)
        experts = pol["experts"][0].tolist()
        raw = pol["raw"][0].tolist()
        weights = [float(v) for v in pol["weights"][0].float().tolist()]
        predicted = pol["pred"][0, : int(pol["npred"][0])].tolist()
        blocked = bool(int(pol["flags"][0]) & 1)
        assert raw == ref["raw_experts"], (t, raw, ref["raw_experts"])
        assert experts == ref["experts"], (t, experts, ref["experts"])
        assert weights == ref["weights"], (t, weights, ref["weights"])
        assert bool(int(pol["flags"][0]) & 2) == ref["sticky_adjusted"], t
        if ref["predicted_experts"] is not None:
            assert predicted == ref["predicted_experts"], (t, predicted, ref["predicted_experts"])
        router._record_route(0, t, experts, weights, raw, blocked, predicted, resident, k, update_state=False)
        if execute:
            assert sorted(resident) == ref["resident_experts"] and k == ref["active_expert_cap"]
            before = {"hits": cache.stats.hits, "misses": cache.stats.misses, "evictions": cache.stats.evictions}
            account_expert_use(cache, 0, experts, H, I, torch.bfloat16)
            after = {"hits": cache.stats.hits, "misses": cache.stats.misses, "evictions": cache.stats.evictions}
            router._after_execution(0, t, experts, before, after)
        prev = experts
    _close(json.loads(json.dumps(router.stats.to_json())), ref_stats)
    assert {str(a): b for a, b in router.dynamic_caps.items()} == json.loads(str(fx["dynamic_caps_json"]))


TIE_CONFIGS = [
    dict(enabled=True, sticky_strength=2.0, semantic_guard=True, min_raw_overlap=2, max_sticky_bonus=0.25,
         max_hot_experts_per_layer=6, exploration_margin=0.25, cache_aware_strength=0.3, predictive_prefetch=True),
    dict(enabled=True, sticky_strength=1.0, semantic_guard=False, max_hot_experts_per_layer=3, exploration_margin=0.5,
         predictive_prefetch=True, prediction_window=5, workload_window=8, sticky_decay=0.5),
    dict(enabled=True, sticky_strength=0.75, semantic_guard=True, min_raw_overlap=3, max_sticky_bonus=1.0,
         cache_aware_strength=0.125, sticky_candidate_margin=1.0),
]


@pytest.mark.parametrize("E,k", [(32, 4), (128, 4), (16, 3), (512, 2)])
@pytest.mark.parametrize("ci", range(len(TIE_CONFIGS)))
def test_device_policy_matches_host_policy_on_ties(E, k, ci):
    from kcapw_klcquant_b200 import RoutingLocalityConfig, StreamedMoERouter

    T = 48
    rng = np.random.default_rng(E * 31 + k * 7 + ci)
    levels = np.array([-1.0, -0.5, 0.0, 0.25, 0.5, 0.75, 1.0], dtype=np.float32)
    lg = levels[rng.integers(0, len(levels), size=(T, E))]
    lg[rng.random((T, E)) < 0.3] += np.float32(0.125)
    bits = orc.f32_to_bf16_bits(lg)
    resident = {int(e) for e in rng.choice(E, size=max(2, E // 4), replace=False)}
    cfg = RoutingLocalityConfig(**TIE_CONFIGS[ci])
    dev_router = StreamedMoERouter(k, 7.0, cfg, matmul_precision="bf16")
    host_router = StreamedMoERouter(k, 7.0, cfg, matmul_precision="bf16", locality_on_device=False)
    pol = dev_router._device_policy(0, _bf16(bits).to(DEV), k, dev_router._resident_mask(resident, E, DEV), 0)
    got = {key: v.cpu() for key, v in pol.items()}
    lf = orc.bf16_bits_to_f32(bits)
    for t in range(T):
        predicted = host_router.predict_experts(0, k)
        raw, experts, scores, blocked = host_router._locality_select(0, torch.from_numpy(lf[t].copy()), k, resident)
        w_bits = orc.softmax_weights_bits(np.asarray(scores, np.float32)[None])[0]
        weights = [float(v) for v in orc.bf16_bits_to_f32(w_bits)]
        assert got["raw"][t].tolist() == raw, (t, got["raw"][t].tolist(), raw)
        assert got["experts"][t].tolist() == experts, (t, got["experts"][t].tolist(), experts)
        assert [float(v) for v in got["weights"][t].float().tolist()] == weights, t
        assert got["pred"][t, : int(got["npred"][t])].tolist() == predicted, (t, predicted)
        assert bool(int(got["flags"][t]) & 1) == blocked, t
        host_router._record_route(0, t, experts, weights, raw, blocked, predicted, resident, k)
    dev_router._sync_host_state(0)
    assert dev_router.sticky_scores[0] == host_router.sticky_scores[0]
    assert list(dev_router.sticky_scores[0]) == list(host_router.sticky_scores[0])  # insertion order too
    assert dev_router.workload_scores[0] == host_router.workload_scores[0]
    assert list(dev_router.recent_history[0]) == list(host_router.recent_history[0])


def test_route_and_route_batch_with_device_policy(tmp_path):
    from kcapw_klcquant_b200 import Mxfp4ExpertStore, RoutingLocalityConfig, StreamedMoERouter
    from kcapw_klcquant_b200 import synthetic as syn
    from tests.golden.make_golden import write_checkpoint

    dims = syn.LayerDims(32, 256, 256, 4)
    layer = syn.make_layer(dims, seed=61)
    write_checkpoint(layer, tmp_path)
    tensors = {n: t.to(DEV) for n, t in syn.dense_tensors(layer).items()}
    x = cases.correlated_hidden(24, 256, 61).to(DEV)
    cfg = RoutingLocalityConfig(enabled=True, sticky_strength=1.5, semantic_guard=True, min_raw_overlap=2,
                                max_hot_experts_per_layer=5, cache_aware_strength=0.2, predictive_prefetch=True)
    resident = {1, 4, 9, 17}
    per_token = StreamedMoERouter(4, 7.0, cfg, matmul_precision="bf16")
    batched = StreamedMoERouter(4, 7.0, cfg, matmul_precision="bf16")
    store = Mxfp4ExpertStore(tmp_path, tmp_path, DEV, dtype=torch.bfloat16, cache_bytes=1 << 40)
    ys, routes = [], []
    for t in range(24):
        y, r = per_token.route(0, x[t], tensors, store, True, t, resident_experts=resident)
        ys.append(y)
        routes.append(r)
    yb, rb = batched.route_batch(0, x, tensors, store, record_stats=True, resident_experts=resident)
    assert rb.indices.tolist() == [r["experts"] for r in routes]
    assert [[float(v) for v in row] for row in rb.weights.float().tolist()] == [r["weights"] for r in routes]
    from tests import parity

    parity.assert_output_close(torch.stack(ys).view(torch.int16).cpu().numpy().view(np.uint16),
                               yb.view(torch.int16).cpu().numpy().view(np.uint16), "route_batch vs route (device policy)")
    # telemetry: the batched records equal the per-token ones (route() adds the cache deltas)
    a, b = per_token.stats.to_json(), batched.stats.to_json()
    for key in ("routed_tokens", "expert_activation_frequency", "route_events"):
        _close(b[key], a[key], key)
    for key in ("guarded_adjustments", "blocked_adjustments", "mean_raw_route_overlap", "prediction_accuracy", "reuse_distance"):
        _close(b["locality"][key], a["locality"][key], key)
    assert per_token.predict_experts(0, 4) == batched.predict_experts(0, 4)
