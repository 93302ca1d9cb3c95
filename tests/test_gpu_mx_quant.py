"""Activation operand of the block-scaled tensor-core path (klc_mx_quantize_rows).

Each bf16 row is split per 32-value block into two E4M3 rows with a shared
E8M0 scale: S = floor(log2 max|x|) - 7, hi = x with the low four mantissa
bits cleared, lo = x - hi, both divided by 2^S and rounded to E4M3
(nearest, ties to even).  The device output must equal this numpy
restatement bit for bit, and hi + lo must reproduce every x within 2^9 of
its block maximum exactly (the exactness the expert GEMMs rely on).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _e4m3_table() -> np.ndarray:
    """Values of the 256 E4M3 codes (NaN codes 0x7F / 0xFF as nan)."""
    v = np.empty(256, np.float64)
    for c in range(256):
        s, e, m = c >> 7, (c >> 3) & 15, c & 7
        if e == 15 and m == 7:
            v[c] = np.nan
            continue
        mag = (m / 8.0) * 2.0**-6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
        v[c] = -mag if s else mag
    return v


E4M3 = _e4m3_table()
_POS = np.arange(0, 127)  # codes 0x00..0x7E: 0 .. 448


def _encode_e4m3(x: np.ndarray) -> np.ndarray:
    """Round to nearest E4M3 (ties to the even code), saturating at 448."""
    a = np.minimum(np.abs(x), 448.0)
    vals = E4M3[_POS]
    idx = np.searchsorted(vals, a)  # vals[idx-1] <= a < vals[idx] (or equal)
    idx = np.clip(idx, 1, len(vals) - 1)
    lo, hi = vals[idx - 1], vals[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & ((idx & 1) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(a == vals[np.clip(idx, 0, len(vals) - 1)], idx, code)
    return (code | np.where(np.signbit(x), 0x80, 0)).astype(np.uint8)  # the sign survives rounding to zero


def _reference_split(xb: np.ndarray):
    """bf16 bit patterns [R, K] -> (q [R, 2, K] u8, scales [R, K/32] u8)."""
    R, K = xb.shape
    blocks = xb.reshape(R, K // 32, 32).astype(np.uint32)
    emax = ((blocks >> 7) & 0xFF).max(axis=2).astype(np.int64)
    S = np.where(emax == 0, 0, emax - 134)
    S = np.clip(S, -126, 126)
    x = (blocks << 16).view(np.float32).astype(np.float64)
    h = ((blocks & 0xFFF0) << 16).view(np.float32).astype(np.float64)
    inv = np.ldexp(1.0, -S)[..., None]
    hi = _encode_e4m3(h * inv)
    lo = _encode_e4m3((x - h) * inv)
    q = np.stack([hi.reshape(R, K), lo.reshape(R, K)], axis=1)
    return q, (S + 127).astype(np.uint8), x.reshape(R, K), S


def _device_split(xb: np.ndarray):
    from kcapw_klcquant_b200 import _lib

    R, K = xb.shape
    x = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).to(DEV)
    q = torch.empty((R, 2, K), dtype=torch.uint8, device=DEV)
    sc = torch.empty((R, K // 32), dtype=torch.uint8, device=DEV)
    _lib.check(_lib.lib().klc_mx_quantize_rows(x.data_ptr(), R, K, q.data_ptr(), sc.data_ptr(), _lib.stream_ptr()))
    return q.cpu().numpy(), sc.cpu().numpy()


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("case", ["normal", "wide_range", "edge"])
def test_split_matches_restatement_and_is_exact_near_block_max(case):
    rng = np.random.default_rng({"normal": 1, "wide_range": 2, "edge": 3}[case])
    R, K = 37, 2880
    if case == "normal":
        xf = rng.standard_normal((R, K)).astype(np.float32)
    elif case == "wide_range":
        xf = (rng.standard_normal((R, K)) * np.exp2(rng.integers(-40, 40, (R, K)))).astype(np.float32)
    else:
        xf = rng.standard_normal((R, K)).astype(np.float32)
        xf[0] = 0.0                                    # all-zero row
        xf[1, :32] = -0.0
        xf[2] = np.float32(3.0e38) * np.sign(rng.standard_normal(K))  # near the bf16 maximum
        xf[3] = np.ldexp(1.0, -133) * rng.integers(1, 100, K)         # bf16 subnormals
        xf[4, ::2] = 1e-30                              # tiny next to O(1) values
    xb = _bf16_bits(xf)
    q, sc = _device_split(xb)
    rq, rsc, x, S = _reference_split(xb)
    np.testing.assert_array_equal(sc, rsc)
    np.testing.assert_array_equal(q, rq)
    # reconstruction: exact within 2^9 of the block maximum (normal bf16 blocks)
    recon = (E4M3[q[:, 0].astype(np.int64)] + E4M3[q[:, 1].astype(np.int64)]).reshape(R, K // 32, 32)
    recon = recon * np.ldexp(1.0, S)[..., None]
    xblk = x.reshape(R, K // 32, 32)
    amax = np.abs(xblk).max(axis=2, keepdims=True)
    near = (np.abs(xblk) >= amax * 2.0**-9) & (amax > np.ldexp(1.0, -120))
    assert np.all(recon[near] == xblk[near])
    far = ~near & (amax > np.ldexp(1.0, -120))
    if far.any():
        assert np.all(np.abs(recon[far] - xblk[far]) <= np.broadcast_to(amax, xblk.shape)[far] * 2.0**-16)


def test_pad_k128_matches_numpy():
    """klc_mxfp4_pad_k128: each row's 16-byte groups copied, zero groups appended up to a multiple of 4."""
    from kcapw_klcquant_b200.mxfp4_expert import pad_k128

    g = torch.Generator().manual_seed(4)
    b = torch.randint(0, 256, (3, 40, 90, 16), generator=g, dtype=torch.uint8)
    out = pad_k128(b.to(DEV)).cpu().numpy()
    want = np.zeros((3, 40, 92, 16), np.uint8)
    want[:, :, :90] = b.numpy()
    np.testing.assert_array_equal(out, want)
    assert pad_k128(torch.zeros((1, 4, 8, 16), dtype=torch.uint8, device=DEV)) is None


def test_scales_tile_layouts():
    """klc_mxfp4_scales_tile: tile 128 equals klc_mxfp4_scales_mx; tile 192 against numpy."""
    from kcapw_klcquant_b200.mxfp4_expert import scales_mx, scales_tile

    g = torch.Generator().manual_seed(6)
    s = torch.randint(0, 256, (2, 400, 90), generator=g, dtype=torch.uint8)
    sd = s.to(DEV)
    np.testing.assert_array_equal(scales_tile(sd, 128).cpu().numpy().reshape(-1), scales_mx(sd).cpu().numpy().reshape(-1))
    got = scales_tile(sd, 192).cpu().numpy()  # [E, tiles, stages, 2, 512]
    E, rows, G = s.shape
    want = np.zeros_like(got)
    sn = s.numpy()
    for t in range(got.shape[1]):
        for m in range(192):
            r = t * 192 + m
            if r >= rows:
                continue
            for g4 in range(G):
                st, kb = divmod(g4, 4)
                c, mm = divmod(m, 128)
                want[:, t, st, c, (mm % 32) * 16 + (mm // 32) * 4 + kb] = sn[:, r, g4]
    np.testing.assert_array_equal(got, want)


def test_bounded_wait_reports_timeout_and_gpu_answers():
    """The bounded mbarrier wait of the tensor-core kernels gives up on a barrier
    nothing arrives on, records KLC_ERR_DEVICE_TIMEOUT at its site, and the GPU
    keeps answering (klc_selftest_wait_timeout, 2e6 cycles ~ 1 ms)."""
    import ctypes

    from kcapw_klcquant_b200 import _lib

    code, where = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.lib().klc_selftest_wait_timeout(2_000_000, ctypes.byref(code), ctypes.byref(where), _lib.stream_ptr()))
    assert code.value == _lib.KLC_ERR_DEVICE_TIMEOUT and where.value == 999
    assert float(torch.arange(8, device=DEV, dtype=torch.float32).sum()) == 28.0
