"""Shared parity metrics and tie-aware routing checks for the tests."""
from __future__ import annotations

import numpy as np

from oracle import moe_oracle as orc

# Output tolerance (bf16 MoE outputs vs the reference's torch path).
# The reference's own fp32 and bf16 paths differ by about 6.5e-3 of max|ref|
# on these synthetic layers; the gate is cosine >= 0.9999 and max-abs
# normalised by max|ref| <= 2e-2.
COSINE_MIN = 0.9999
NORM_MAX_ABS = 2e-2


def output_metrics(got_bits: np.ndarray, ref_bits: np.ndarray) -> dict:
    a = orc.bf16_bits_to_f32(got_bits).astype(np.float64).ravel()
    b = orc.bf16_bits_to_f32(ref_bits).astype(np.float64).ravel()
    diff = np.abs(a - b)
    scale = max(np.abs(b).max(), 1e-30)
    cos = float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))
    return {
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "norm_max_abs": float(diff.max() / scale) if diff.size else 0.0,
        "cosine": cos,
        "bit_equal_frac": float(np.mean(np.asarray(got_bits) == np.asarray(ref_bits))),
    }


def assert_output_close(got_bits, ref_bits, label: str = "") -> dict:
    m = output_metrics(got_bits, ref_bits)
    assert m["cosine"] >= COSINE_MIN, (label, m)
    assert m["norm_max_abs"] <= NORM_MAX_ABS, (label, m)
    return m


def ulp_distance_bf16(a_bits, b_bits) -> np.ndarray:
    """Distance in bf16 ulps between two bit arrays (sign-magnitude ordered)."""

    def ordered(u):
        u = np.asarray(u, dtype=np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u & 0x7FFF)

    return np.abs(ordered(a_bits) - ordered(b_bits))


def check_selection(logits_bits: np.ndarray, got_idx: np.ndarray, k: int, strict_tie_order: bool = True) -> int:
    """Assert that each row of ``got_idx`` is a valid top-k of the bf16 logits.

    Valid means: every expert strictly above the k-th value is selected, the
    rest come from the class tied at the k-th value, and the order is by
    descending logit with ties by lower index (any tie order when
    ``strict_tie_order`` is False, as for the reference's CPU topk).  Returns the number of rows that
    had an exact tie at the boundary.
    """
    lg = orc.bf16_bits_to_f32(logits_bits)
    classes = orc.topk_tie_classes(lg, k)
    ties = 0
    for t, (must, maybe) in enumerate(classes):
        row = [int(v) for v in got_idx[t]]
        assert len(set(row)) == k, (t, row)
        assert must <= set(row), (t, row, must)
        assert set(row) - must <= maybe, (t, row, must, maybe)
        if len(maybe) > k - len(must):
            ties += 1
        vals = lg[t, row]
        for a in range(k - 1):
            assert vals[a] > vals[a + 1] or (vals[a] == vals[a + 1] and (row[a] < row[a + 1] or not strict_tie_order)), (t, row, vals)
    return ties


def same_selection_modulo_ties(logits_bits: np.ndarray, ref_idx: np.ndarray, got_idx: np.ndarray, k: int) -> None:
    """The reference's and our selection agree except inside an exact tie class."""
    lg = orc.bf16_bits_to_f32(logits_bits)
    for t, (must, maybe) in enumerate(orc.topk_tie_classes(lg, k)):
        r, g = set(int(v) for v in ref_idx[t]), set(int(v) for v in got_idx[t])
        assert must <= r and must <= g, (t, r, g, must)
        assert r - must <= maybe and g - must <= maybe, (t, r, g, maybe)
