"""The host-side routing policy and telemetry against the reference's own route().

Fixtures (tests/golden/locality_*.npz, made by tests/golden/make_golden.py)
record, for correlated token sequences, the reference's per-token routing
dicts and its final ``RouterStats.to_json()`` with ``RoutingLocalityConfig``
enabled (sticky bonus, semantic guard, hot-expert mask, cache-aware bonus,
dynamic active-expert cap, predictive prefetch) and with the default config.

Stage-isolated (the reference's logits are the input, as SURVEY's routing
policy prescribes): the policy steps of ``StreamedMoERouter.route``
(``_locality_select``, ``_record_route``, ``_after_execution``) run on the CPU
in route()'s order, the softmax is the oracle's, and the expert-cache lookups
are accounted by the same function the store uses.  Selections, weights,
predictions, caps and the whole ``to_json()`` must equal the reference's.
"""
from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.golden import cases


def _close(a, b, path="$"):
    if isinstance(a, dict) and isinstance(b, dict):
        assert set(a) == set(b), (path, sorted(set(a) ^ set(b)))
        for k in a:
            _close(a[k], b[k], f"{path}.{k}")
    elif isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        assert len(a) == len(b), (path, len(a), len(b))
        for i, (x, y) in enumerate(zip(a, b)):
            _close(x, y, f"{path}[{i}]")
    elif isinstance(a, float) or isinstance(b, float):
        assert a is not None and b is not None, (path, a, b)
        assert math.isclose(float(a), float(b), rel_tol=1e-9, abs_tol=1e-12), (path, a, b)
    else:
        assert a == b, (path, a, b)


@pytest.mark.parametrize("name", list(cases.LOCALITY_CASES))
def test_locality_policy_and_stats_match_reference(golden_dir, name):
    from kcapw_klcquant_b200 import RoutingLocalityConfig, StreamedMoERouter
    from kcapw_klcquant_b200.mxfp4_expert import DenseMatrixCache, account_expert_use

    E, H, I, k_top, T, seed, execute, cfg_kw = cases.LOCALITY_CASES[name]
    fx = np.load(golden_dir / f"locality_{name}.npz")
    ref_routes = json.loads(str(fx["routes_json"]))
    ref_stats = json.loads(str(fx["stats_json"]))
    cfg = RoutingLocalityConfig(**cfg_kw) if cfg_kw is not None else None
    router = StreamedMoERouter(k_top, 7.0, cfg, matmul_precision="bf16")
    cache = DenseMatrixCache(1 << 40)  # the fixtures' reference store holds every matrix (no evictions)
    logits = orc.bf16_bits_to_f32(fx["logits"])
    prev: list[int] = []
    for t in range(T):
        ref = ref_routes[t]
        lg = logits[t]
        k = router._effective_expert_count(0, E)
        resident = cases.resident_set(t, prev) if cfg is not None else None
        if router.locality_config.enabled:
            # host policy: torch.topk on the host logits, ties resolved as in the reference
            raw, experts, scores, blocked = router._locality_select(0, torch.from_numpy(lg.copy()), k, resident or set())
        else:
            # device selection: descending value, lower index on exact ties (the kernel's rule)
            sel, vals = orc.select_topk(lg[None], k)
            raw = [int(e) for e in sel[0]]
            experts, scores, blocked = raw, list(vals[0]), False
        assert raw == ref["raw_experts"], (t, raw, ref["raw_experts"])
        assert experts == ref["experts"], (t, experts, ref["experts"])
        w_bits = orc.softmax_weights_bits(np.asarray(scores, np.float32)[None])[0]
        weights = [float(v) for v in orc.bf16_bits_to_f32(w_bits)]
        assert weights == ref["weights"], (t, weights, ref["weights"])
        predicted, resident_sorted, adjusted = router._record_route(0, t, experts, weights, raw, blocked, None, resident, k)
        assert adjusted == ref["sticky_adjusted"], (t, ref)
        if ref["predicted_experts"] is not None:  # the bias-only dict has no prediction key (:323-329)
            assert predicted == ref["predicted_experts"], (t, predicted, ref)
        if execute:
            assert resident_sorted == ref["resident_experts"] and k == ref["active_expert_cap"]
            before = {"hits": cache.stats.hits, "misses": cache.stats.misses, "evictions": cache.stats.evictions}
            account_expert_use(cache, 0, experts, H, I, torch.bfloat16)
            after = {"hits": cache.stats.hits, "misses": cache.stats.misses, "evictions": cache.stats.evictions}
            router._after_execution(0, t, experts, before, after)
        prev = experts
    _close(json.loads(json.dumps(router.stats.to_json())), ref_stats)
    assert {str(a): b for a, b in router.dynamic_caps.items()} == json.loads(str(fx["dynamic_caps_json"]))
