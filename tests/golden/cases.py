"""Route-fixture cases shared by the fixture generator and the tests."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from kcapw_klcquant_b200 import synthetic as syn

HERE = Path(__file__).resolve().parent

# Route cases: name -> (E, H, I, k, T, seed, zipf, tie_rows, capture_intermediates)
ROUTE_CASES = {
    "c0_e32_h2880_t8": (32, 2880, 2880, 4, 8, 0, None, 0, False),
    "c1_e128_h2880_t8": (128, 2880, 2880, 4, 8, 1, None, 0, False),
    "mini_e16_h256_t32": (16, 256, 256, 4, 32, 11, None, 0, True),
    "mini_zipf_e32_h128_t64": (32, 128, 128, 4, 64, 12, 1.1, 0, False),
    "mini_e8_h64_t5_k2": (8, 64, 64, 2, 5, 13, None, 0, True),
    "mini_e8_h128_i192_t6": (8, 128, 192, 4, 6, 14, None, 0, True),
    "tie_e16_h64_t24": (16, 64, 64, 4, 24, 15, None, 4, False),
    # full layout with more than 12 rows per expert: the tensor-core path's 64-row tiles
    "mid_e8_h2880_t48": (8, 2880, 2880, 4, 48, 16, None, 0, False),
    "mid_zipf_e16_h2880_t64": (16, 2880, 2880, 4, 64, 17, 1.1, 0, False),
}

# Cases at the full GPT-OSS layout (H = I = 2880): routing and outputs checked on
# a token subsample by the CPU oracle tests (each token touches ~25 M weights).
FULL_LAYOUT_CASES = [n for n, spec in ROUTE_CASES.items() if spec[1] >= 2880]
SMALL_LAYOUT_CASES = [n for n in ROUTE_CASES if n not in FULL_LAYOUT_CASES]

# Locality-policy cases (the reference's route() with RoutingLocalityConfig on):
# name -> (E, H, I, k, T, seed, execute_experts, config kwargs or None for the default config)
LOCALITY_CASES = {
    "loc_full_e16_h256_t32": (16, 256, 256, 4, 32, 51, True,
                              dict(enabled=True, sticky_strength=2.0, semantic_guard=True, min_raw_overlap=2, max_sticky_bonus=0.25,
                                   max_hot_experts_per_layer=6, exploration_margin=0.25, cache_aware_strength=0.3,
                                   predictive_prefetch=True, dynamic_active_expert_cap=True, active_experts_per_token_cap=3,
                                   min_active_experts_per_token=2, max_active_experts_per_token=4)),
    "loc_noguard_e16_h256_t32": (16, 256, 256, 4, 32, 52, False,
                                 dict(enabled=True, sticky_strength=1.0, semantic_guard=False, max_hot_experts_per_layer=4,
                                      exploration_margin=0.5, predictive_prefetch=True)),
    "loc_default_e16_h256_t12": (16, 256, 256, 4, 12, 53, True, None),
}


def correlated_hidden(T: int, H: int, seed: int) -> torch.Tensor:
    """bf16 [T, H] token sequence whose neighbours are correlated (x_t = 0.8 x_{t-1} + 0.6 noise),
    so sticky experts carry over between positions."""
    g = torch.Generator().manual_seed(seed + 31337)
    x = torch.randn((T, H), generator=g, dtype=torch.float32)
    for t in range(1, T):
        x[t] = 0.8 * x[t - 1] + 0.6 * x[t]
    return x.to(torch.bfloat16)


def resident_set(t: int, previous_experts: list[int]) -> set[int]:
    """Experts a cache-aware caller reports resident at position t: the previous
    token's experts plus experts 0 and 1."""
    return set(int(e) for e in previous_experts) | {0, 1}


def tie_layer(layer: dict[str, torch.Tensor], tie_rows: int, seed: int) -> None:
    """Copy router rows so several experts share a logit (exact ties at the top-k boundary)."""
    if not tie_rows:
        return
    key = "model.layers.0.mlp.router.weight"
    w = layer[key].clone()
    g = torch.Generator().manual_seed(seed + 3)
    src = int(torch.randint(0, w.shape[0], (1,), generator=g))
    for r in range(tie_rows):
        w[(src + 1 + 2 * r) % w.shape[0]] = w[src]
    layer[key] = w



def load_route_case(name: str, with_experts: bool = True):
    """Fixture arrays plus the regenerated inputs of one route case."""
    fx = dict(np.load(HERE / f"route_{name}.npz"))
    E, H, I, k, T, seed, zipf_m, tie_rows = (int(v) for v in fx["meta"])
    zipf = None if zipf_m < 0 else zipf_m / 1000.0
    dims = syn.LayerDims(E, H, I, k)
    layer = syn.make_layer(dims, seed, zipf=zipf)
    tie_layer(layer, tie_rows, seed)
    x = syn.make_hidden(T, H, seed)
    return fx, dims, layer, x


def bits(t: torch.Tensor) -> np.ndarray:
    """uint16 bit patterns of a bf16 tensor (or uint8/int arrays unchanged)."""
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy()
