"""CPU oracle for the KLCquant MoE block — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference computes on its MoE hot
path.  It is the checker used by ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``; the product
(``kcapw_klcquant_b200``) never imports it and has no CPU fallback.

Parity pin: the reference has no tests of its own, so the oracle is pinned
against fixtures in ``tests/golden/`` that were produced by running the
reference's own functions on seeded synthetic inputs
(``tests/golden/make_golden.py``).  ``tests/test_oracle_golden.py`` checks every
function below against those fixtures.

bf16 is emulated with uint16 bit patterns; rounding is round-to-nearest-even,
as ``torch`` does it (NaN -> 0x7FC0).
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(a) -> np.ndarray:
    """Round fp32 values to bf16 (nearest-even) and return the uint16 bit patterns."""
    f = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0) | ((u >> 16).astype(np.uint16) & np.uint16(0x8000)), rounded)
    return rounded


def bf16_bits_to_f32(bits) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(bits, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    """fp32 -> bf16 -> fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# ---------------------------------------------------------------------------
# MXFP4 dequant (klcquant mxfp4_expert.py:17-34, 357-379)
# ---------------------------------------------------------------------------

# E2M1 magnitudes by nibble; nibble 8 is -0.0 (mxfp4_expert.py:17-34).
FP4_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float64
)


def dequantize_mxfp4_exact(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Exact values of an MXFP4 matrix as float32, returned in [in, out] order.

    blocks uint8 [out, G, 16], scales uint8 [out, G].  Within a byte the low
    nibble is the even K index and the high nibble the odd one
    (mxfp4_expert.py:375-376); each value is ``FP4[nibble] * 2**(scale-127)``
    (:367, :377), and the [out, G*32] matrix is transposed to [in, out]
    (:378-379).  E2M1 values have two significant bits, so every product is
    exact in float32 (subnormals included) or overflows to +/-inf exactly where
    the exact value exceeds the float32 range.
    """
    blocks = np.asarray(blocks, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.uint8)
    if blocks.shape[:-1] != scales.shape:
        raise ValueError(f"MXFP4 block/scale shape mismatch: {blocks.shape=} {scales.shape=}")
    return np.ascontiguousarray(dequantize_mxfp4_out_in(blocks, scales).T)


def dequantize_mxfp4_out_in(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Exact float32 MXFP4 values in the stored [out, in] order (no transpose)."""
    blocks = np.asarray(blocks, dtype=np.uint8)
    out_dim, groups, packed = blocks.shape
    idx = (np.asarray(scales, dtype=np.int32) << 8)[..., None] | blocks
    return _byte_pair_table()[idx].reshape(out_dim, groups * packed * 2)


_PAIRS: np.ndarray | None = None


def _byte_pair_table() -> np.ndarray:
    """[scale*256 + byte] -> (value of low nibble, value of high nibble), float32."""
    global _PAIRS
    if _PAIRS is None:
        e = np.arange(256, dtype=np.int32)[:, None] - 127
        with np.errstate(over="ignore"):
            per_scale = np.ldexp(FP4_VALUES.astype(np.float32)[None, :], e).astype(np.float32)  # [256, 16]
        byte = np.arange(256)
        _PAIRS = np.stack([per_scale[:, byte & 0x0F], per_scale[:, byte >> 4]], axis=-1).reshape(-1, 2)
    return _PAIRS


def dequantize_mxfp4_bits(blocks: np.ndarray, scales: np.ndarray, dtype: str) -> np.ndarray:
    """Bit patterns of ``dequantize_mxfp4_matrix(blocks, scales, dtype)``.

    dtype is ``"bf16"``, ``"f16"`` or ``"f32"``.  The exact value is rounded
    once to the target type; overflow gives +/-inf and the sign of zero is kept.
    """
    exact = dequantize_mxfp4_exact(blocks, scales)
    if dtype == "f32":
        return exact.view(np.uint32)
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return exact.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return f32_to_bf16_bits(exact)
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# Router (klcquant streamed_moe_router.py:257-284)
# ---------------------------------------------------------------------------


def router_logits_bits(x_bits: np.ndarray, w_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """bf16 logits of ``F.linear(hidden, W_r, b_r)`` (streamed_moe_router.py:269).

    Restated as an fp32-accumulated dot product plus the bias, rounded once to
    bf16.  The reference's CPU GEMV blocks its accumulation differently, so a
    small fraction of logits can differ by one bf16 ulp; parity tests account
    for that explicitly.
    """
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    b = bf16_bits_to_f32(b_bits).astype(np.float64)
    acc = (x @ w.T).astype(np.float32) + b.astype(np.float32)
    return f32_to_bf16_bits(acc)


def select_topk(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Top-k of fp32 logits per row, descending, ties broken by the lower index.

    The reference calls ``torch.topk(logits.float(), k)`` (:271, :273) whose
    tie order is unspecified; this oracle (and the CUDA kernel) fixes it to
    "lower expert index first".
    """
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    k = min(k, E)
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -logits.astype(np.float64)), axis=-1)[:, :k]
    return order.astype(np.int32), np.take_along_axis(logits, order, axis=1)


def softmax_weights_bits(scores: np.ndarray) -> np.ndarray:
    """``softmax(fp32 selected scores).to(bf16)`` (:281-282)."""
    s = np.asarray(scores, dtype=np.float32)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp((s - m).astype(np.float32)).astype(np.float32)
    return f32_to_bf16_bits(e / e.sum(axis=-1, keepdims=True, dtype=np.float32))


def topk_tie_classes(logits: np.ndarray, k: int) -> list[tuple[set[int], set[int]]]:
    """Per row: (experts that must be selected, experts of which some may be selected).

    With an exact tie at the k boundary any member of the tied class is a
    valid pick; the harness accepts any of them.
    """
    logits = np.asarray(logits, dtype=np.float32)
    out = []
    for row in logits:
        srt = np.sort(row)[::-1]
        kth = srt[k - 1]
        must = set(np.nonzero(row > kth)[0].tolist())
        maybe = set(np.nonzero(row == kth)[0].tolist())
        out.append((must, maybe))
    return out


# ---------------------------------------------------------------------------
# Dispatch: counting-sort permutation (no counterpart in the reference, which
# loops over one token at a time; defined here as a stable sort)
# ---------------------------------------------------------------------------


def moe_permute(indices: np.ndarray, experts: int, pad: int = 1) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Group (token, slot) pairs by expert.

    Returns ``(rows, counts, offsets)``: ``rows[p]`` is the flat pair id
    ``token*k + slot`` stored at padded position ``p`` (or -1 in padding),
    ``counts[e]`` the pairs routed to expert ``e`` and ``offsets[e]`` the first
    padded position of expert ``e`` (each group padded to a multiple of
    ``pad``).  Pairs of one expert keep token-major, slot-minor order (a stable
    sort of the flat expert ids).
    """
    flat = np.asarray(indices, dtype=np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=experts).astype(np.int32)
    padded = ((counts + pad - 1) // pad) * pad
    offsets = np.zeros(experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(padded)
    rows = np.full(int(offsets[-1]), -1, dtype=np.int32)
    order = np.argsort(flat, kind="stable")
    start = 0
    for e in range(experts):
        c = int(counts[e])
        rows[offsets[e] : offsets[e] + c] = order[start : start + c]
        start += c
    return rows, counts, offsets


# ---------------------------------------------------------------------------
# Experts (klcquant streamed_moe_router.py:483-529)
# ---------------------------------------------------------------------------


def apply_gate(gu: np.ndarray, limit: float = 7.0, alpha: float = 1.702) -> np.ndarray:
    """Clamped SwiGLU of interleaved gate/up rows (:524-529).

    gate = even columns clamped above at ``limit``; up = odd columns clamped to
    [-limit, limit]; result ``(up + 1) * gate * sigmoid(alpha * gate)`` in fp32.
    """
    gu = np.asarray(gu, dtype=np.float32)
    gate = np.minimum(gu[..., 0::2], np.float32(limit))
    up = np.clip(gu[..., 1::2], np.float32(-limit), np.float32(limit))
    with np.errstate(over="ignore"):
        sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-(gate * np.float32(alpha))))).astype(np.float32)
    return ((up + np.float32(1.0)) * (gate * sig)).astype(np.float32)


def expert_forward(
    x_bits: np.ndarray,
    w_gate_up: np.ndarray,
    b_gate_up_bits: np.ndarray,
    w_down: np.ndarray,
    b_down_bits: np.ndarray,
    precision: str = "fp32",
    limit: float = 7.0,
    alpha: float = 1.702,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """One expert on rows ``x`` [n, H]: returns (gu, gated, out) in fp32.

    ``w_gate_up`` is the dense [H, 2I] matrix and ``w_down`` [I, H] (bf16-exact
    values as float32).  'fp32' mirrors :505, :511 (fp32 GEMV + fp32 bias);
    'bf16' mirrors :502-503, :507-509 (bf16 product rounded, then fp32 bias).
    """
    x = bf16_bits_to_f32(x_bits)
    bgu = bf16_bits_to_f32(b_gate_up_bits)
    bd = bf16_bits_to_f32(b_down_bits)
    # fp32 GEMV/GEMM with fp32 accumulation (BLAS), as the reference's torch CPU matmuls
    if precision == "bf16":
        gu = round_bf16(x @ w_gate_up) + bgu
        gated = apply_gate(gu, limit, alpha)
        out = round_bf16(round_bf16(gated) @ w_down) + bd
    else:
        gu = (x @ w_gate_up) + bgu
        gated = apply_gate(gu, limit, alpha)
        out = (gated @ w_down) + bd
    return gu.astype(np.float32), gated, out.astype(np.float32)


def combine_bits(outs: np.ndarray, weight_bits: np.ndarray) -> np.ndarray:
    """bf16 weighted combine in selection order (:497, :512-513).

    ``output`` starts at bf16 zero; for each selected expert in top-k order
    ``output += out.to(bf16) * w`` with every product and sum rounded to bf16.
    outs fp32 [..., k, H]; weight_bits uint16 [..., k].
    """
    outs = np.asarray(outs, dtype=np.float32)
    w = bf16_bits_to_f32(weight_bits)
    acc = np.zeros(outs.shape[:-2] + outs.shape[-1:], dtype=np.float32)
    for s in range(outs.shape[-2]):
        prod = round_bf16(round_bf16(outs[..., s, :]) * w[..., s, None])
        acc = round_bf16(acc + prod)
    return f32_to_bf16_bits(acc)


class DenseExperts:
    """Lazily dequantized dense expert matrices (float32, bf16-exact values)."""

    def __init__(self, gu_blocks, gu_scales, d_blocks, d_scales, max_cached: int | None = None):
        self.gu_blocks, self.gu_scales = np.asarray(gu_blocks), np.asarray(gu_scales)
        self.d_blocks, self.d_scales = np.asarray(d_blocks), np.asarray(d_scales)
        self.cache: dict[int, tuple[np.ndarray, np.ndarray]] = {}
        # at the 120B layout one dense expert is ~100 MB of float32: a bound keeps
        # host memory flat when a check walks many experts once each
        self.max_cached = max_cached

    def get(self, e: int) -> tuple[np.ndarray, np.ndarray]:
        if e not in self.cache:
            if self.max_cached is not None and len(self.cache) >= self.max_cached:
                self.cache.pop(next(iter(self.cache)))
            # E2M1 x E8M0 values are exact in bf16 (same exponent range as fp32,
            # two significant bits), so the float32 values equal the bf16 matrix
            # the reference caches.  Stored as [in, out] views of [out, in] arrays.
            gu = dequantize_mxfp4_out_in(self.gu_blocks[e], self.gu_scales[e]).T
            dn = dequantize_mxfp4_out_in(self.d_blocks[e], self.d_scales[e]).T
            self.cache[e] = (gu, dn)
        return self.cache[e]


def moe_layer(
    x_bits: np.ndarray,
    indices: np.ndarray,
    weight_bits: np.ndarray,
    experts: DenseExperts,
    b_gate_up_bits: np.ndarray,
    b_down_bits: np.ndarray,
    precision: str = "fp32",
    limit: float = 7.0,
    alpha: float = 1.702,
    return_intermediates: bool = False,
):
    """Expert execution + combine for a batch of tokens with given routing.

    Mirrors ``_execute_mxfp4_experts`` (:483-522) one token at a time, grouped
    by expert for speed (the arithmetic per (token, expert) pair is the same).
    Returns the bf16 output bits [T, H] (and per-pair fp32 gu/gated/out).
    """
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    indices = np.asarray(indices, dtype=np.int64)
    T, k = indices.shape
    H = x_bits.shape[1]
    gu_all = gated_all = None
    outs = np.zeros((T, k, H), dtype=np.float32)
    inter = {}
    for e in np.unique(indices):
        tok, slot = np.nonzero(indices == e)
        wgu, wd = experts.get(int(e))
        gu, gated, out = expert_forward(x_bits[tok], wgu, b_gate_up_bits[e], wd, b_down_bits[e], precision, limit, alpha)
        outs[tok, slot] = out
        if return_intermediates:
            if gu_all is None:
                gu_all = np.zeros((T, k, gu.shape[1]), np.float32)
                gated_all = np.zeros((T, k, gated.shape[1]), np.float32)
            gu_all[tok, slot] = gu
            gated_all[tok, slot] = gated
    y = combine_bits(outs, weight_bits)
    if return_intermediates:
        inter = {"gu": gu_all, "gated": gated_all, "out": outs}
        return y, inter
    return y


def bias_only_bits(indices: np.ndarray, weight_bits: np.ndarray, b_down_bits: np.ndarray) -> np.ndarray:
    """``execute_experts=False`` path (:317-329): sum of bf16 down biases times weights.

    ``torch.sum(selected * weights[:, None], dim=0)`` in bf16: the products are
    rounded to bf16, the sum over k is accumulated in fp32 and rounded once.
    """
    b = bf16_bits_to_f32(np.asarray(b_down_bits)[np.asarray(indices)])  # [T, k, H]
    w = bf16_bits_to_f32(weight_bits)[..., None]
    prod = round_bf16(b * w)
    return f32_to_bf16_bits(prod.sum(axis=-2, dtype=np.float32))


# ---------------------------------------------------------------------------
# RMSNorm (klcquant streamed_attention.py:27-28)
# ---------------------------------------------------------------------------


def rms_norm_bits(x_bits: np.ndarray, w_bits: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """``x * rsqrt(mean(x.float()**2) + eps).to(bf16) * weight``, all products bf16."""
    x = bf16_bits_to_f32(x_bits)
    w = bf16_bits_to_f32(w_bits)
    ms = np.mean(x.astype(np.float32) * x.astype(np.float32), axis=-1, keepdims=True, dtype=np.float32)
    r = round_bf16((np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32))
    return f32_to_bf16_bits(round_bf16(round_bf16(x * r) * w))


# ---------------------------------------------------------------------------
# Runtime dequantizer (klcquant runtime_dequantizer.py:30-52,
# adaptive_quantizer.py:183-213, tensor_pruner.py:62-69)
# ---------------------------------------------------------------------------


def unpack_lowbit(packed: np.ndarray, bits: int, numel: int) -> np.ndarray:
    """Signed integers from the reference's packed low-bit formats.

    q1: 8 values per byte, LSB first, bit set -> +1 else -1.  q2: 4 per byte,
    value = field - 2.  q4: 2 per byte (low nibble first), value = field - 8.
    q3: 8 values per 3 bytes (little-endian 24-bit word, 3-bit fields LSB
    first), value = field - 4.
    """
    if bits not in (1, 2, 3, 4):
        raise ValueError("unpack_lowbit only supports q1, q2, q3 and q4")
    p = np.asarray(packed, dtype=np.uint8).reshape(-1).astype(np.int64)
    offset = 1 << (bits - 1)
    if bits in (1, 2, 4):
        per = 8 // bits
        mask = (1 << bits) - 1
        fields = np.stack([(p >> (i * bits)) & mask for i in range(per)], axis=1).reshape(-1)[:numel]
        if bits == 1:
            return np.where(fields > 0, 1, -1).astype(np.int8)
        return (fields - offset).astype(np.int8)
    if p.size % 3:
        p = np.concatenate([p, np.zeros(3 - p.size % 3, dtype=np.int64)])
    words = p.reshape(-1, 3)
    w24 = words[:, 0] | (words[:, 1] << 8) | (words[:, 2] << 16)
    fields = np.stack([(w24 >> (i * 3)) & 7 for i in range(8)], axis=1).reshape(-1)[:numel]
    return (fields - offset).astype(np.int8)


def _to_dtype_bits(v: np.ndarray, dtype: str) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    if dtype == "f32":
        return v.view(np.uint32)
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return v.astype(np.float16).view(np.uint16)
    return f32_to_bf16_bits(v)


def runtime_dequantize_bits(mode: str, data: np.ndarray, scale: np.ndarray | None, shape, dtype: str, bits: int = 16, packed: bool = False) -> np.ndarray:
    """``RuntimeDequantizer.dequantize`` (runtime_dequantizer.py:30-52) as bit patterns.

    fp16: ``data.to(dtype)``; packed q1-q4: ``unpack_lowbit`` then
    ``q.float() * scale.float()`` rounded once to ``dtype``; unpacked q8/q16:
    the same product on the stored integers.
    """
    numel = int(np.prod(shape))
    if mode == "fp16":
        v = np.asarray(data).astype(np.float32)
        return _to_dtype_bits(v, dtype).reshape(shape)
    if scale is None:
        raise ValueError("quantized tensor has no scale tensor")
    q = unpack_lowbit(data, bits, numel) if packed else np.asarray(data).reshape(-1)
    v = q.astype(np.float32) * np.asarray(scale, dtype=np.float32).reshape(-1)[0]
    return _to_dtype_bits(v, dtype).reshape(shape)


def reconstruct_pruned_bits(values_f32: np.ndarray, indices: np.ndarray, shape, dtype: str) -> np.ndarray:
    """``reconstruct_pruned`` (tensor_pruner.py:62-69): zeros with values scattered at flat indices."""
    numel = int(np.prod(shape))
    out = np.zeros(numel, dtype=np.float32)
    out[np.asarray(indices, dtype=np.int64)] = np.asarray(values_f32, dtype=np.float32)
    return _to_dtype_bits(out, dtype).reshape(shape)
