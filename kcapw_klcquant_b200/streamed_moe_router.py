"""Drop-in ``StreamedMoERouter`` running the MoE block on B200 kernels.

Same constructor, ``route()`` signature and returned dict keys as klcquant's
streamed_moe_router.py (``StreamedMoERouter`` :238-529,
``RoutingLocalityConfig`` :12-35, ``RouterStats`` :38-235), plus a batched
``route_batch()`` for many tokens per call.

Per call the device does all MoE math: router logits + top-k + softmax
(``klc_router_topk``), dispatch, MXFP4 expert GEMMs with the clamped SwiGLU,
and the bf16 combine (``klc_moe_experts`` / ``klc_moe_forward``).  The host
keeps what the reference keeps on the host: the routing statistics, and --
only when ``RoutingLocalityConfig.enabled`` -- the locality policy (sticky /
cache-aware bias and the semantic guard, :331-394), evaluated on the E logits
read back from the device, as the reference evaluates it through
``.tolist()`` / ``.item()``.
"""
from __future__ import annotations

import math
from collections import Counter, deque
from dataclasses import dataclass, field

import torch

from . import _lib
import ctypes

from .moe import MoeLayer, RouteBatch, as_bf16, rms_norm, workspace
from .mxfp4_expert import Mxfp4ExpertStore


@dataclass
class RoutingLocalityConfig:
    """Locality-aware routing knobs (same fields and defaults as the reference, :12-35)."""

    enabled: bool = False
    sticky_strength: float = 0.0
    sticky_decay: float = 0.92
    semantic_guard: bool = False
    sticky_candidate_margin: float = 0.50
    max_sticky_bonus: float = 0.25
    min_raw_overlap: int = 2
    max_hot_experts_per_layer: int = 0
    active_experts_per_token_cap: int = 0
    exploration_margin: float = 0.25
    cache_aware_strength: float = 0.0
    predictive_prefetch: bool = False
    prediction_window: int = 16
    workload_window: int = 64
    dynamic_active_expert_cap: bool = False
    min_active_experts_per_token: int = 1
    max_active_experts_per_token: int = 0
    cap_eviction_pressure_threshold: float = 0.50
    cap_hit_rate_expand_threshold: float = 0.65
    thrash_evictions_per_activation: float = 0.35
    thrash_reuse_density: float = 0.15
    thrash_active_growth: float = 0.25


def _percentile_summary(values: list[int]) -> dict:
    if not values:
        return {"count": 0, "mean": None, "p50": None, "p90": None, "max": None}
    v = sorted(values)
    n = len(v)
    return {"count": n, "mean": sum(v) / n, "p50": v[int(0.50 * (n - 1))], "p90": v[int(0.90 * (n - 1))], "max": v[-1]}


@dataclass
class RouterStats:
    """Host-side routing telemetry with the reference's JSON schema (:38-235)."""

    expert_hits: Counter = field(default_factory=Counter)
    routed_tokens: int = 0
    route_events: list[dict] = field(default_factory=list)
    last_seen_position: dict[tuple[int, int], int] = field(default_factory=dict)
    reuse_distances: list[int] = field(default_factory=list)
    active_by_position: dict[int, set[tuple[int, int]]] = field(default_factory=dict)
    route_entropies: list[float] = field(default_factory=list)
    cache_delta_events: list[dict] = field(default_factory=list)
    cap_events: list[dict] = field(default_factory=list)
    guarded_adjustments: int = 0
    blocked_adjustments: int = 0
    raw_overlap_total: int = 0
    route_count: int = 0

    def record_route(self, layer_idx, position, experts, weights, raw_experts, adjusted, predicted_experts=None,
                     resident_experts=None, active_cap=None, blocked_adjustment=False) -> None:
        self.routed_tokens += 1
        self.route_count += 1
        entropy = -sum(float(w) * math.log(max(float(w), 1e-12)) for w in weights)
        self.route_entropies.append(entropy)
        overlap = len({int(e) for e in experts} & {int(e) for e in raw_experts})
        self.raw_overlap_total += overlap
        self.guarded_adjustments += int(bool(adjusted))
        self.blocked_adjustments += int(bool(blocked_adjustment))
        active = self.active_by_position.setdefault(int(position), set())
        reuse = []
        for e in experts:
            key = (int(layer_idx), int(e))
            self.expert_hits[key] += 1
            active.add(key)
            prev = self.last_seen_position.get(key)
            if prev is not None:
                d = int(position) - prev
                self.reuse_distances.append(d)
                reuse.append(d)
            self.last_seen_position[key] = int(position)
        self.route_events.append({
            "position": int(position),
            "layer": int(layer_idx),
            "experts": [int(e) for e in experts],
            "raw_experts": [int(e) for e in raw_experts],
            "predicted_experts": [int(e) for e in (predicted_experts or [])],
            "resident_experts": [int(e) for e in (resident_experts or [])],
            "weights": [float(w) for w in weights],
            "route_entropy": entropy,
            "reuse_distances": reuse,
            "sticky_adjusted": adjusted,
            "blocked_locality_adjustment": blocked_adjustment,
            "raw_route_overlap": overlap,
            "active_expert_cap": active_cap,
        })

    def record_cache_delta(self, layer_idx, position, experts, before, after) -> None:
        self.cache_delta_events.append({
            "position": int(position),
            "layer": int(layer_idx),
            "experts": [int(e) for e in experts],
            **{k: int(after.get(k, 0)) - int(before.get(k, 0)) for k in ("hits", "misses", "evictions")},
        })

    def record_cap_event(self, layer_idx, position, old_cap, new_cap, reason, hits, misses, evictions) -> None:
        if old_cap == new_cap:
            return
        self.cap_events.append({"position": int(position), "layer": int(layer_idx), "old_cap": int(old_cap), "new_cap": int(new_cap),
                                "reason": reason, "hits": int(hits), "misses": int(misses), "evictions": int(evictions)})

    def _entropy(self) -> float:
        total = sum(self.expert_hits.values())
        if not total:
            return 0.0
        return -sum((c / total) * math.log(max(c / total, 1e-12)) for c in self.expert_hits.values())

    def _hit_eviction_corr(self) -> dict:
        ev = self.cache_delta_events
        if not ev:
            return {"sample_count": 0, "correlation": None}
        h = [float(x.get("hits", 0)) for x in ev]
        e = [float(x.get("evictions", 0)) for x in ev]
        mh, me = sum(h) / len(h), sum(e) / len(e)
        cov = sum((a - mh) * (b - me) for a, b in zip(h, e))
        den = math.sqrt(sum((a - mh) ** 2 for a in h) * sum((b - me) ** 2 for b in e))
        return {"sample_count": len(h), "correlation": cov / den if den > 0 else None}

    def _prediction_accuracy(self) -> dict:
        rows = [x for x in self.route_events if x.get("predicted_experts")]
        if not rows:
            return {"sample_count": 0, "mean_precision": None, "mean_recall": None, "exact_match_rate": None}
        prec, rec, exact = [], [], 0
        for x in rows:
            a, p = set(x.get("experts", [])), set(x.get("predicted_experts", []))
            o = len(a & p)
            prec.append(o / max(len(p), 1))
            rec.append(o / max(len(a), 1))
            exact += int(a == p)
        return {"sample_count": len(rows), "mean_precision": sum(prec) / len(prec), "mean_recall": sum(rec) / len(rec),
                "exact_match_rate": exact / len(rows)}

    def to_json(self) -> dict:
        activations = sum(self.expert_hits.values())
        unique = len(self.expert_hits)
        evictions = sum(int(x.get("evictions", 0)) for x in self.cache_delta_events)
        rows = [{"position": int(p), "active_expert_count": len(s)} for p, s in sorted(self.active_by_position.items())]
        counts = [r["active_expert_count"] for r in rows]
        growth = (counts[-1] - counts[0]) / max(counts[0], 1) if len(counts) >= 2 else 0.0
        reuse_density = len(self.reuse_distances) / max(activations, 1)
        ev_per_act = evictions / max(activations, 1)
        ev_per_1k = 1000.0 * evictions / max(self.routed_tokens, 1)
        thrash = ev_per_act >= 0.35 and (reuse_density <= 0.15 or growth >= 0.25 or ev_per_1k >= 1000.0 or unique >= max(activations * 0.50, 1))
        return {
            "routed_tokens": self.routed_tokens,
            "expert_activation_frequency": {str(k): v for k, v in self.expert_hits.most_common()},
            "locality": {
                "total_expert_activations": activations,
                "unique_expert_activations": unique,
                "reuse_density": reuse_density,
                "reuse_distance": _percentile_summary(self.reuse_distances),
                "routing_entropy_mean": sum(self.route_entropies) / max(len(self.route_entropies), 1),
                "routing_entropy_distribution": self._entropy(),
                "active_expert_set_size_over_time": rows,
                "active_expert_set_growth": growth,
                "cache_evictions_observed": evictions,
                "evictions_per_activation": ev_per_act,
                "evictions_per_1k_routed_tokens": ev_per_1k,
                "expert_thrash_mode": thrash,
                "cache_hit_eviction_correlation": self._hit_eviction_corr(),
                "prediction_accuracy": self._prediction_accuracy(),
                "dynamic_cap_events": self.cap_events[:500],
                "guarded_adjustments": int(self.guarded_adjustments),
                "blocked_adjustments": int(self.blocked_adjustments),
                "mean_raw_route_overlap": self.raw_overlap_total / max(self.route_count, 1),
            },
            "route_events": self.route_events[:500],
            "cache_delta_events": self.cache_delta_events[:500],
        }


class StreamedMoERouter:
    """MoE block with the reference's API (streamed_moe_router.py:238-529), executed by libklcmoe."""

    def __init__(self, experts_per_token: int = 4, swiglu_limit: float = 7.0, locality_config: RoutingLocalityConfig | None = None,
                 matmul_precision: str = "fp32", expert_path: str = "auto", locality_on_device: bool = True) -> None:
        if matmul_precision not in _lib.PRECISION_CODE:
            raise ValueError(f"matmul_precision must be one of {sorted(_lib.PRECISION_CODE)}")
        self.experts_per_token = experts_per_token
        self.swiglu_limit = swiglu_limit
        self.alpha = 1.702
        self._stats = RouterStats()
        # route_batch() routings on their way to the host: (copy-done event, layer, first position, k,
        # pinned expert ids, pinned weights); recorded, in call order, whenever the stats are read
        self._pending: list[tuple] = []
        self.locality_config = locality_config or RoutingLocalityConfig()
        self.matmul_precision = matmul_precision
        self.expert_path = expert_path
        self.sticky_scores: dict[int, dict[int, float]] = {}
        self.workload_scores: dict[int, dict[int, float]] = {}
        self.recent_history: dict[int, deque[int]] = {}
        self.dynamic_caps: dict[int, int] = {}
        self._layers: dict[tuple, MoeLayer] = {}
        # locality policy on the GPU (klc_locality_route): per-layer state buffers on the device; the
        # host dicts above are then rebuilt from them only when predict_experts() is called
        self.locality_on_device = bool(locality_on_device)
        self._loc_states: dict[int, torch.Tensor] = {}

    @property
    def stats(self) -> RouterStats:
        """The routing telemetry (reference ``RouterStats``), with every pending
        route_batch() routing recorded first."""
        self._flush_pending()
        return self._stats

    def _flush_pending(self) -> None:
        while self._pending:
            done, layer_idx, position, k, ids_h, ws_h, loc = self._pending.pop(0)
            done.synchronize()
            ids, ws = ids_h.tolist(), ws_h.float().tolist()
            if loc is None:
                for t, (e, w) in enumerate(zip(ids, ws)):
                    self._stats.record_route(layer_idx, position + t, e, w, e, False, active_cap=k)
                continue
            raw_h, pred_h, npred_h, flags_h, resident = loc
            raws, preds, npreds, flags = raw_h.tolist(), pred_h.tolist(), npred_h.tolist(), flags_h.tolist()
            for t, (e, w) in enumerate(zip(ids, ws)):
                self._stats.record_route(layer_idx, position + t, e, w, raws[t], e != raws[t], predicted_experts=preds[t][: npreds[t]],
                                         resident_experts=resident, active_cap=k, blocked_adjustment=bool(flags[t] & 1))

    # ------------------------------------------------------------------
    # device layer cache
    # ------------------------------------------------------------------
    def _moe_layer(self, layer_idx: int, tensors: dict[str, torch.Tensor], store: Mxfp4ExpertStore, k: int) -> MoeLayer:
        p = f"model.layers.{layer_idx}.mlp"
        packed = store.layer(layer_idx)
        srcs = (tensors[f"{p}.router.weight"], tensors[f"{p}.router.bias"], tensors[f"{p}.experts.gate_up_proj_bias"], tensors[f"{p}.experts.down_proj_bias"])
        key = (int(layer_idx), k, id(packed)) + tuple((t.data_ptr(), t._version) for t in srcs)
        layer = self._layers.get(key)
        if layer is None:
            self._layers = {kk: v for kk, v in self._layers.items() if kk[0] != int(layer_idx)}
            layer = MoeLayer(packed, *srcs, top_k=k, swiglu_limit=self.swiglu_limit, alpha=self.alpha, path=self.expert_path)
            self._layers[key] = layer
        return layer

    # ------------------------------------------------------------------
    # route(): one token, reference semantics
    # ------------------------------------------------------------------
    def route(self, layer_idx: int, hidden: torch.Tensor, tensors: dict[str, torch.Tensor], expert_store: Mxfp4ExpertStore | None = None,
              execute_experts: bool = True, position: int = 0, predicted_experts: list[int] | None = None,
              resident_experts: set[int] | None = None) -> tuple[torch.Tensor, dict]:
        self._flush_pending()  # earlier route_batch() routings are recorded before this token
        p = f"model.layers.{layer_idx}.mlp"
        w_r, b_r = tensors[f"{p}.router.weight"], tensors[f"{p}.router.bias"]
        if not hidden.is_cuda:
            raise ValueError("route() runs on the GPU; hidden must be a CUDA tensor")
        dev = hidden.device
        E, H = int(w_r.shape[0]), int(hidden.shape[-1])
        k = self._effective_expert_count(layer_idx, E)
        x = as_bf16(hidden.reshape(1, H), dev)
        w_dev, b_dev = as_bf16(w_r, dev), as_bf16(b_r, dev)
        idx = torch.empty((1, k), dtype=torch.int32, device=dev)
        wts = torch.empty((1, k), dtype=torch.bfloat16, device=dev)
        logits = torch.empty((1, E), dtype=torch.bfloat16, device=dev)
        cfg = self.locality_config
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().klc_router_topk(x.data_ptr(), 1, H, w_dev.data_ptr(), b_dev.data_ptr(), E, k, None,
                                                  idx.data_ptr(), wts.data_ptr(), logits.data_ptr(), _lib.stream_ptr()))
        gu_b = tensors.get(f"{p}.experts.gate_up_proj_bias")
        dn_b = tensors.get(f"{p}.experts.down_proj_bias")
        if not cfg.enabled or self.locality_on_device:
            return self._route_on_device(layer_idx, hidden, x, tensors, expert_store, execute_experts, position, predicted_experts,
                                         resident_experts, logits, idx, wts, k, gu_b, dn_b)
        # host locality policy (locality_on_device=False): the logits come to the host first
        raw_experts, experts, scores, blocked = self._locality_select(layer_idx, logits[0].float().cpu(), k, resident_experts or set())
        sc = torch.tensor(scores, dtype=torch.float32, device=dev).reshape(1, k)
        idx = torch.tensor([experts], dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().klc_select_softmax(sc.data_ptr(), 1, k, k, 1, None, wts.data_ptr(), _lib.stream_ptr()))
        weights_list = [float(v) for v in wts[0].float().tolist()]
        predicted, resident, adjusted_flag = self._record_route(layer_idx, position, experts, weights_list, raw_experts, blocked,
                                                                predicted_experts, resident_experts, k)
        norms_list = None
        y = None
        store_path = execute_experts and expert_store is not None
        if store_path and gu_b is not None and dn_b is not None:
            layer = self._moe_layer(layer_idx, tensors, expert_store, k)
            y, norms = layer.experts_forward(x, idx, wts, precision=self.matmul_precision, return_norms=True)
            norms_list = norms[0].tolist()
        elif not store_path and dn_b is not None:
            y = self._bias_only(x, tensors, p, idx, wts, k)
        return self._finish_route(layer_idx, hidden, expert_store, execute_experts, position, experts, weights_list, raw_experts,
                                  predicted, resident, adjusted_flag, k, y, norms_list, gu_b, dn_b, tensors, p)

    def _bias_only(self, x: torch.Tensor, tensors, p: str, idx: torch.Tensor, wts: torch.Tensor, k: int) -> torch.Tensor:
        dev = x.device
        H = int(x.shape[-1])
        db = as_bf16(tensors[f"{p}.experts.down_proj_bias"], dev)
        y = torch.empty((1, H), dtype=torch.bfloat16, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().klc_moe_bias_only(db.data_ptr(), 1, H, k, idx.data_ptr(), wts.data_ptr(), y.data_ptr(), _lib.stream_ptr()))
        return y

    def _route_on_device(self, layer_idx, hidden, x, tensors, expert_store, execute_experts, position, predicted_experts,
                         resident_experts, logits, idx, wts, k, gu_b, dn_b):
        """route() with the selection on the device (plain top-k, or the locality kernel): the
        experts (or the bias-only path) are launched on the device routing right away, and the
        routing, the locality outputs and the expert norms come back in one copy; the host-side
        steps (statistics, policy bookkeeping, expert-cache accounting) then run in the
        reference's order on those values."""
        p = f"model.layers.{layer_idx}.mlp"
        dev = x.device
        E = int(logits.shape[1])
        loc = self.locality_config.enabled
        pol = None
        if loc:
            pol = self._device_policy(layer_idx, logits, k, self._resident_mask(resident_experts, E, dev), 0)
            idx, wts = pol["experts"], pol["weights"]
        store_path = execute_experts and expert_store is not None
        y, norms = None, None
        if store_path and gu_b is not None and dn_b is not None:
            layer = self._moe_layer(layer_idx, tensors, expert_store, k)
            y, norms = layer.experts_forward(x, idx, wts, precision=self.matmul_precision, return_norms=True)
        elif not store_path and dn_b is not None:
            y = self._bias_only(x, tensors, p, idx, wts, k)
        parts = [idx.reshape(-1).double(), wts.reshape(-1).double()]
        if loc:
            parts += [pol["raw"].reshape(-1).double(), pol["pred"].reshape(-1).double(), pol["npred"].double(), pol["flags"].double()]
        if norms is not None:
            parts.append(norms.reshape(-1).double())
        host = torch.cat(parts).cpu().tolist()  # the one synchronisation of the call
        experts = [int(v) for v in host[:k]]
        weights_list = [float(v) for v in host[k:2 * k]]
        at = 2 * k
        blocked = False
        if loc:
            raw_experts = [int(v) for v in host[at:at + k]]
            npred = int(host[at + 2 * k])
            if predicted_experts is None:
                predicted_experts = [int(v) for v in host[at + k:at + k + npred]]
            blocked = bool(int(host[at + 2 * k + 1]) & 1)
            at += 2 * k + 2
        else:
            raw_experts = list(experts)
        norms_list = None
        if norms is not None:
            flat = host[at:at + 2 * k]
            norms_list = [[flat[2 * i], flat[2 * i + 1]] for i in range(k)]
        # the device kernel already advanced the layer's locality state
        predicted, resident, adjusted_flag = self._record_route(layer_idx, position, experts, weights_list, raw_experts, blocked,
                                                                predicted_experts, resident_experts, k, update_state=not loc)
        return self._finish_route(layer_idx, hidden, expert_store, execute_experts, position, experts, weights_list, raw_experts,
                                  predicted, resident, adjusted_flag, k, y, norms_list, gu_b, dn_b, tensors, p)

    def _finish_route(self, layer_idx, hidden, expert_store, execute_experts, position, experts, weights_list, raw_experts,
                      predicted, resident, adjusted_flag, k, y, norms_list, gu_b, dn_b, tensors, p):
        """The route() dict and the expert-store bookkeeping, in the reference's order (:303-329)."""
        if execute_experts and expert_store is not None:
            before = self._cache_snapshot(expert_store)
            expert_store.protect_experts(layer_idx, experts)
            if gu_b is None or dn_b is None:
                output, route = torch.zeros_like(hidden), {"experts": experts, "weights": weights_list, "mode": "mxfp4_missing_bias"}
            else:
                expert_store.note_expert_use(layer_idx, experts)  # the reference's two load_expert_matrix calls per expert
                output = y.reshape(hidden.shape).to(hidden.dtype)
                route = {
                    "experts": experts,
                    "weights": weights_list,
                    "mode": "mxfp4_expert_matmul",
                    "expert_logs": [
                        {"expert": int(e), "routing_weight": weights_list[i], "gate_up_norm": float(norms_list[i][0]),
                         "output_norm": float(norms_list[i][1])}
                        for i, e in enumerate(experts)
                    ],
                }
            self._after_execution(layer_idx, position, experts, before, self._cache_snapshot(expert_store))
            route["raw_experts"] = raw_experts
            route["predicted_experts"] = [int(v) for v in predicted]
            route["resident_experts"] = resident
            route["sticky_adjusted"] = adjusted_flag
            route["active_expert_cap"] = k
            return output, route
        if dn_b is None:
            return torch.zeros_like(hidden), {"experts": experts, "weights": weights_list, "mode": "router_only"}
        return y.reshape(hidden.shape).to(hidden.dtype), {
            "experts": experts,
            "raw_experts": raw_experts,
            "weights": weights_list,
            "mode": "bias_only_moe",
            "sticky_adjusted": adjusted_flag,
        }

    # ------------------------------------------------------------------
    # route_batch(): many tokens per call (new, additive API)
    # ------------------------------------------------------------------
    def route_batch(self, layer_idx: int, hidden: torch.Tensor, tensors: dict[str, torch.Tensor], expert_store: Mxfp4ExpertStore,
                    *, return_logits: bool = False, return_norms: bool = False, residual: torch.Tensor | None = None,
                    record_stats: bool = False, position: int = 0,
                    next_norm: tuple[torch.Tensor, float] | None = None,
                    resident_experts: set[int] | None = None) -> tuple[torch.Tensor, RouteBatch]:
        """Route and execute T tokens at once: hidden bf16 [T, H] -> (output [T, H], RouteBatch).

        With locality disabled this equals calling ``route()`` per token.  With
        locality enabled the policy runs on the device (klc_locality_route) over
        the tokens in order, continuing the layer's sticky / workload state as
        T consecutive route() calls would, with one active-expert count for the
        whole batch (the dynamic cap adapts between calls) and one
        ``resident_experts`` set for every token; the expert-cache deltas and
        the cap are not updated per token.  With ``record_stats`` the routing is
        copied asynchronously into pinned host buffers on the call's stream (no
        synchronisation here) and recorded as positions ``position ..
        position+T-1`` when the statistics are next read (``router.stats``) or
        ``route()`` runs.  ``next_norm=(weight, eps)`` adds the next layer's input
        RMSNorm of the output (``RouteBatch.normed``), fused into the combine
        when locality is off.
        """
        p = f"model.layers.{layer_idx}.mlp"
        E = int(tensors[f"{p}.router.weight"].shape[0])
        k = self._effective_expert_count(layer_idx, E)
        layer = self._moe_layer(layer_idx, tensors, expert_store, k)
        loc = None
        if self.locality_config.enabled:
            if not self.locality_on_device:
                raise ValueError("route_batch() with locality needs the device policy (locality_on_device=True); use route() otherwise")
            x = as_bf16(hidden, layer.device)
            T = int(x.shape[0])
            logits = torch.empty((T, E), dtype=torch.bfloat16, device=layer.device)
            ridx = torch.empty((T, k), dtype=torch.int32, device=layer.device)
            rw = torch.empty((T, k), dtype=torch.bfloat16, device=layer.device)
            with torch.cuda.device(layer.device):
                _lib.check(_lib.lib().klc_router_topk(x.data_ptr(), T, int(x.shape[1]), layer.router_weight.data_ptr(),
                                                      layer.router_bias.data_ptr(), E, k, None, ridx.data_ptr(), rw.data_ptr(),
                                                      logits.data_ptr(), _lib.stream_ptr(layer.device)))
            pol = self._device_policy(layer_idx, logits, k, self._resident_mask(resident_experts, E, layer.device), 0)
            y, norms = layer.experts_forward(x, pol["experts"], pol["weights"], precision=self.matmul_precision,
                                             return_norms=return_norms, residual=residual)
            normed = rms_norm(y, next_norm[0], float(next_norm[1])) if next_norm is not None else None
            rb = RouteBatch(pol["experts"], pol["weights"], logits=logits if return_logits else None, norms=norms, normed=normed)
            if record_stats:
                loc = [pol["raw"], pol["pred"], pol["npred"], pol["flags"]]
        else:
            y, rb = layer.forward(hidden, precision=self.matmul_precision, return_logits=return_logits, return_norms=return_norms,
                                  residual=residual, next_norm=next_norm)
        if record_stats:
            def pinned(t: torch.Tensor) -> torch.Tensor:
                h = torch.empty(tuple(t.shape), dtype=t.dtype, pin_memory=True)
                h.copy_(t, non_blocking=True)
                return h

            ids_h, ws_h = pinned(rb.indices), pinned(rb.weights)
            if loc is not None:
                loc = [pinned(t) for t in loc] + [sorted(int(v) for v in (resident_experts or set()))]
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(rb.indices.device))
            self._pending.append((done, layer_idx, position, k, ids_h, ws_h, loc))
        return y, rb

    # ------------------------------------------------------------------
    # host-side steps of route(), in the reference's order (:270-315)
    # ------------------------------------------------------------------
    def _locality_select(self, layer_idx: int, logits: torch.Tensor, k: int,
                         resident_experts: set[int]) -> tuple[list[int], list[int], list[float], bool]:
        """Raw top-k, locality bias, adjusted top-k and the semantic guard on one
        token's fp32 logits [E] (a host tensor): (raw experts, experts, scores for
        the softmax, blocked).  The top-k selections use torch.topk on the host
        tensor, as the reference does (:271-273), so exact ties resolve as there."""
        raw_experts = [int(e) for e in torch.topk(logits, k=k).indices.tolist()]
        adjusted = self._apply_locality_bias(layer_idx, logits, resident_experts)
        adj_top = [int(e) for e in torch.topk(adjusted, k=k).indices.tolist()]
        experts, scores, blocked = self._guarded_expert_selection(logits, adjusted, raw_experts, adj_top, k)
        return raw_experts, experts, scores, blocked

    def _record_route(self, layer_idx: int, position: int, experts: list[int], weights: list[float], raw_experts: list[int],
                      blocked: bool, predicted_experts: list[int] | None, resident_experts: set[int] | None, k: int,
                      update_state: bool = True):
        """Statistics and sticky / workload state after a selection (:285-302):
        returns (predicted experts, sorted resident experts, sticky_adjusted).
        ``update_state=False`` when the device policy already updated the state."""
        adjusted_flag = experts != raw_experts
        predicted = predicted_experts if predicted_experts is not None else self.predict_experts(layer_idx, k)
        resident = sorted(int(v) for v in (resident_experts or set()))
        self._stats.record_route(layer_idx, position, experts, weights, raw_experts, adjusted_flag,
                                predicted_experts=[int(v) for v in predicted], resident_experts=resident, active_cap=k,
                                blocked_adjustment=blocked)
        if update_state:
            self._update_sticky_scores(layer_idx, experts, weights)
            self._update_workload_scores(layer_idx, experts, weights)
        return predicted, resident, adjusted_flag

    # ------------------------------------------------------------------
    # locality policy on the device (klc_locality_route)
    # ------------------------------------------------------------------
    def _loc_config(self) -> "_lib.KlcLocalityConfig":
        cfg = self.locality_config
        return _lib.KlcLocalityConfig(
            float(cfg.sticky_strength), float(cfg.sticky_candidate_margin), float(cfg.max_sticky_bonus), float(cfg.exploration_margin),
            float(cfg.cache_aware_strength), float(cfg.sticky_decay), float(cfg.workload_window), int(bool(cfg.semantic_guard)),
            int(cfg.min_raw_overlap), int(cfg.max_hot_experts_per_layer), int(cfg.prediction_window), int(bool(cfg.predictive_prefetch)),
            int(self.experts_per_token))

    def _loc_state(self, layer_idx: int, dev: torch.device, E: int) -> torch.Tensor:
        """The layer's policy state on the device (zero = empty dicts), created on first use."""
        st = self._loc_states.get(layer_idx)
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().klc_locality_state_bytes(E, int(self.locality_config.prediction_window), ctypes.byref(n)))
        if st is None:
            st = torch.zeros(int(n.value), dtype=torch.uint8, device=dev)
            self._loc_states[layer_idx] = st
        elif st.device != dev or st.numel() != int(n.value):
            raise ValueError(f"layer {layer_idx}: locality state was made for another device or expert count")
        return st

    @staticmethod
    def _resident_mask(resident_experts: set[int] | None, E: int, dev: torch.device) -> torch.Tensor | None:
        if not resident_experts:
            return None
        ids = sorted(int(v) for v in resident_experts)
        if ids[0] < 0 or ids[-1] >= E:
            raise IndexError(f"resident expert ids must be in [0, {E})")
        mask = torch.zeros(E, dtype=torch.uint8)
        mask[ids] = 1
        return mask.to(dev, non_blocking=True)

    def _device_policy(self, layer_idx: int, logits: torch.Tensor, k: int, resident: torch.Tensor | None,
                       resident_stride: int) -> dict[str, torch.Tensor]:
        """klc_locality_route over bf16 logits [T, E]: the raw / adjusted / guarded selections, weights,
        predictions and flags of every token, the layer's state advanced token by token."""
        dev = logits.device
        T, E = int(logits.shape[0]), int(logits.shape[1])
        st = self._loc_state(layer_idx, dev, E)
        out = {
            "experts": torch.empty((T, k), dtype=torch.int32, device=dev),
            "weights": torch.empty((T, k), dtype=torch.bfloat16, device=dev),
            "raw": torch.empty((T, k), dtype=torch.int32, device=dev),
            "pred": torch.empty((T, k), dtype=torch.int32, device=dev),
            "npred": torch.empty((T,), dtype=torch.int32, device=dev),
            "flags": torch.empty((T,), dtype=torch.uint8, device=dev),
        }
        cfg = self._loc_config()
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().klc_locality_route(
                ctypes.byref(cfg), logits.contiguous().data_ptr(), T, E, k, _lib.ptr(resident), int(resident_stride), st.data_ptr(),
                st.numel(), out["experts"].data_ptr(), out["weights"].data_ptr(), out["raw"].data_ptr(), out["pred"].data_ptr(),
                out["npred"].data_ptr(), out["flags"].data_ptr(), _lib.stream_ptr(dev)))
        return out

    def _sync_host_state(self, layer_idx: int) -> None:
        """Rebuild the host dicts (insertion order included) from the layer's device state."""
        st = self._loc_states.get(layer_idx)
        if st is None:
            return
        E = (st.numel() - 64 - 4 * max(int(self.locality_config.prediction_window), 1)) // 32
        raw = st.cpu().numpy()
        head = raw[:64].view("<i4")
        hist_len, hist_head = int(head[4]), int(head[5])
        body = raw[64:]
        sticky = body[: 8 * E].view("<f8")
        work = body[8 * E:16 * E].view("<f8")
        s_at = body[16 * E:24 * E].view("<i8")
        w_at = body[24 * E:32 * E].view("<i8")
        W = max(int(self.locality_config.prediction_window), 1)
        hist = body[32 * E:32 * E + 4 * W].view("<i4")
        self.sticky_scores[layer_idx] = {int(e): float(sticky[e]) for e in sorted(range(E), key=lambda e: s_at[e]) if s_at[e] != 0}
        self.workload_scores[layer_idx] = {int(e): float(work[e]) for e in sorted(range(E), key=lambda e: w_at[e]) if w_at[e] != 0}
        self.recent_history[layer_idx] = deque((int(hist[(hist_head + i) % W]) for i in range(hist_len)), maxlen=W)

    def _after_execution(self, layer_idx: int, position: int, experts: list[int], before: dict, after: dict) -> None:
        """Cache-delta statistics and the dynamic active-expert cap (:307-309)."""
        self._stats.record_cache_delta(layer_idx, position, experts, before, after)
        self._adapt_active_cap(layer_idx, position, before, after)

    # ------------------------------------------------------------------
    # locality policy (host side, reference semantics :331-476)
    # ------------------------------------------------------------------
    def _apply_locality_bias(self, layer_idx: int, logits: torch.Tensor, resident_experts: set[int]) -> torch.Tensor:
        """Sticky bonus, hot-expert mask and cache-aware bonus (:331-363), with the
        reference's fp32 tensor arithmetic for the thresholds and bonuses."""
        cfg = self.locality_config
        if not cfg.enabled:
            return logits
        adjusted = logits.clone()
        raw_k = min(self.experts_per_token, logits.numel())
        raw_top = torch.topk(logits, k=raw_k)
        floor = raw_top.values[-1] - abs(float(cfg.sticky_candidate_margin))  # fp32, as the reference
        scores = self.sticky_scores.get(layer_idx, {})
        if scores and cfg.sticky_strength > 0:
            eligible = [int(e) for e in scores if logits[int(e)] >= floor]
            if eligible:
                ids = torch.tensor(eligible, dtype=torch.long)
                bonus = torch.tensor([scores[e] for e in eligible], dtype=logits.dtype) * float(cfg.sticky_strength)
                if cfg.semantic_guard and cfg.max_sticky_bonus > 0:
                    bonus = torch.clamp(bonus, max=float(cfg.max_sticky_bonus))
                adjusted[ids] += bonus
        if cfg.max_hot_experts_per_layer > 0 and len(scores) >= cfg.max_hot_experts_per_layer:
            hot = set(int(e) for e in sorted(scores, key=scores.get, reverse=True)[: cfg.max_hot_experts_per_layer])
            top_ids = raw_top.indices.tolist()
            allowed = hot | {int(e) for e in top_ids[: max(1, self.experts_per_token // 2)]}
            mask = torch.ones_like(adjusted, dtype=torch.bool)
            mask[list(allowed)] = False
            adjusted[mask] -= abs(float(cfg.exploration_margin))
        if resident_experts and cfg.cache_aware_strength > 0:
            ids = torch.tensor(sorted(resident_experts), dtype=torch.long)
            threshold = torch.max(logits) - abs(float(cfg.exploration_margin))
            eligible = ids[logits[ids] >= threshold]
            if eligible.numel() > 0:
                adjusted[eligible] += float(cfg.cache_aware_strength)
        return adjusted

    def _guarded_expert_selection(self, logits, adjusted_logits, raw_experts, adjusted_experts, k):
        cfg = self.locality_config
        if not (cfg.enabled and cfg.semantic_guard):
            return [int(e) for e in adjusted_experts], [float(adjusted_logits[int(e)]) for e in adjusted_experts], False
        raw = [int(e) for e in raw_experts[:k]]
        selected = [int(e) for e in adjusted_experts[:k]]
        raw_set, sel_set = set(raw), set(selected)
        need = min(max(int(cfg.min_raw_overlap), 0), k)
        blocked = False
        while len(raw_set & sel_set) < need:
            missing = [e for e in raw if e not in sel_set]
            replaceable = [e for e in selected if e not in raw_set]
            if not missing or not replaceable:
                break
            evict = min(replaceable, key=lambda e: float(adjusted_logits[e]))
            selected[selected.index(evict)] = missing[0]
            sel_set = set(selected)
            blocked = True
        selected = sorted(selected, key=lambda e: float(adjusted_logits[e]), reverse=True)
        return selected, [float(logits[e]) for e in selected], blocked

    def _update_sticky_scores(self, layer_idx: int, experts: list[int], weights: list[float]) -> None:
        cfg = self.locality_config
        if not cfg.enabled:
            return
        scores = self.sticky_scores.setdefault(layer_idx, {})
        for e in list(scores):
            scores[e] *= float(cfg.sticky_decay)
            if scores[e] < 1e-4:
                del scores[e]
        for e, w in zip(experts, weights):
            scores[int(e)] = scores.get(int(e), 0.0) + float(w)
        if cfg.max_hot_experts_per_layer > 0 and len(scores) > cfg.max_hot_experts_per_layer * 2:
            keep = set(sorted(scores, key=scores.get, reverse=True)[: cfg.max_hot_experts_per_layer])
            for e in list(scores):
                if e not in keep:
                    del scores[e]

    def _update_workload_scores(self, layer_idx: int, experts: list[int], weights: list[float]) -> None:
        cfg = self.locality_config
        scores = self.workload_scores.setdefault(layer_idx, {})
        decay = 1.0 - 1.0 / max(float(cfg.workload_window), 1.0)
        for e in list(scores):
            scores[e] *= decay
            if scores[e] < 1e-4:
                del scores[e]
        hist = self.recent_history.setdefault(layer_idx, deque(maxlen=max(int(cfg.prediction_window), 1)))
        for e, w in zip(experts, weights):
            scores[int(e)] = scores.get(int(e), 0.0) + float(w)
            hist.append(int(e))

    def predict_experts(self, layer_idx: int, limit: int | None = None) -> list[int]:
        cfg = self.locality_config
        if not cfg.enabled or not cfg.predictive_prefetch:
            return []
        if self.locality_on_device and layer_idx in self._loc_states:
            self._sync_host_state(layer_idx)
        scores: Counter[int] = Counter()
        for e, v in self.workload_scores.get(layer_idx, {}).items():
            scores[int(e)] += float(v)
        for e, v in self.sticky_scores.get(layer_idx, {}).items():
            scores[int(e)] += float(v) * 0.75
        for e in self.recent_history.get(layer_idx, []):
            scores[int(e)] += 0.50
        if not scores:
            return []
        n = max(int(limit or self.experts_per_token), 1)
        return [int(e) for e, _ in scores.most_common(n)]

    def _effective_expert_count(self, layer_idx: int, expert_count: int) -> int:
        cfg = self.locality_config
        k = min(self.experts_per_token, expert_count)
        if cfg.enabled and cfg.active_experts_per_token_cap > 0:
            k = min(k, int(cfg.active_experts_per_token_cap))
        if cfg.enabled and cfg.dynamic_active_expert_cap:
            base = cfg.active_experts_per_token_cap or self.experts_per_token
            cur = self.dynamic_caps.setdefault(layer_idx, min(max(base, cfg.min_active_experts_per_token), cfg.max_active_experts_per_token or self.experts_per_token))
            k = min(k, cur)
        return max(k, 1)

    def _adapt_active_cap(self, layer_idx: int, position: int, before: dict, after: dict) -> None:
        cfg = self.locality_config
        if not (cfg.enabled and cfg.dynamic_active_expert_cap):
            return
        old = self.dynamic_caps.setdefault(layer_idx, cfg.active_experts_per_token_cap or self.experts_per_token)
        hits = int(after.get("hits", 0)) - int(before.get("hits", 0))
        misses = int(after.get("misses", 0)) - int(before.get("misses", 0))
        evictions = int(after.get("evictions", 0)) - int(before.get("evictions", 0))
        total = hits + misses
        hit_rate, pressure = hits / max(total, 1), evictions / max(total, 1)
        lo, hi = max(int(cfg.min_active_experts_per_token), 1), int(cfg.max_active_experts_per_token or self.experts_per_token)
        new, reason = old, ""
        if pressure >= float(cfg.cap_eviction_pressure_threshold) and old > lo:
            new, reason = old - 1, "eviction_pressure"
        elif evictions == 0 and hit_rate >= float(cfg.cap_hit_rate_expand_threshold) and old < hi:
            new, reason = old + 1, "stable_high_hit_rate"
        if new != old:
            self.dynamic_caps[layer_idx] = new
            self._stats.record_cap_event(layer_idx, position, old, new, reason, hits, misses, evictions)

    @staticmethod
    def _cache_snapshot(expert_store) -> dict:
        s = expert_store.cache.stats
        return {"hits": s.hits, "misses": s.misses, "evictions": s.evictions}
