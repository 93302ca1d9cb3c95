"""CPU-side checks of the C ABI: the library loads, exports every declared
symbol, and validates arguments on the host before touching a GPU."""
from __future__ import annotations

import ctypes
import re

import pytest

from kcapw_klcquant_b200 import _lib
from tests.conftest import REPO

HEADER = REPO / "include" / "klc_moe.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(klc_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 15, names
    for n in names:
        assert hasattr(L, n), f"libklcmoe.so does not export {n}"
    assert L.klc_version() >= 1


def test_python_signatures_cover_header():
    names = set(declared_functions())
    assert names - {"klc_last_error"} <= set(_lib.SIGNATURES), names - set(_lib.SIGNATURES)


def _status_and_msg(st):
    return st, _lib.lib().klc_last_error().decode()


def test_host_validation_without_gpu():
    L = _lib.lib()
    st, msg = _status_and_msg(L.klc_mxfp4_dequant(None, None, -1, 3, None, 0, None))
    assert st == _lib.KLC_ERR_INVALID and "negative" in msg
    st, msg = _status_and_msg(L.klc_mxfp4_dequant(None, None, 0, 0, None, 0, None))
    assert st == _lib.KLC_OK  # empty matrix is a no-op
    st, msg = _status_and_msg(L.klc_router_topk(None, 4, 2880, None, None, 128, 9, None, None, None, None, None))
    assert st == _lib.KLC_ERR_INVALID and "k" in msg
    st, msg = _status_and_msg(L.klc_runtime_dequant(7, None, 0, None, None, 0, 4, 10, None, 0, None))
    assert st == _lib.KLC_ERR_INVALID
    st, msg = _status_and_msg(L.klc_runtime_dequant(1, None, 0, None, None, 0, 4, 10, ctypes.c_void_p(16), 0, None))
    assert st == _lib.KLC_ERR_INVALID and "scale" in msg
    fake = ctypes.c_void_p(256)
    st, msg = _status_and_msg(L.klc_moe_combine(fake, fake, fake, 4, 9, 2880, None, fake, None))
    assert st == _lib.KLC_ERR_INVALID and "k <= 8" in msg
    st, msg = _status_and_msg(L.klc_moe_combine_rmsnorm(fake, fake, fake, 4, 2, 2880, None, None, 1e-5, fake, fake, None))
    assert st == _lib.KLC_ERR_INVALID and "null" in msg
    st, msg = _status_and_msg(L.klc_moe_combine_rmsnorm(fake, fake, fake, 4, 2, 2884, None, fake, 1e-5, fake, fake, None))
    assert st == _lib.KLC_ERR_INVALID and "sizes" in msg
    st, msg = _status_and_msg(L.klc_moe_combine_rmsnorm(fake, fake, fake, 4, 2, 2880, None, fake, 1e-5, fake,
                                                        ctypes.c_void_p(264), None))
    assert st == _lib.KLC_ERR_INVALID and "aligned" in msg
    st, msg = _status_and_msg(L.klc_moe_combine_rmsnorm(None, None, None, 0, 2, 2880, None, None, 1e-5, None, None, None))
    assert st == _lib.KLC_OK  # no tokens: nothing to do
    d = _lib.KlcDims(4, 2880, 2880, 128, 4, _lib.PATH_CODE["auto"])
    st, msg = _status_and_msg(L.klc_moe_forward_rmsnorm(ctypes.byref(d), None, fake, None, 0, fake, fake, fake, None, None,
                                                        None, None, 1e-5, fake, fake, 0, None))
    assert st == _lib.KLC_ERR_INVALID and "RMSNorm" in msg


def test_check_maps_invalid_to_value_error():
    L = _lib.lib()
    with pytest.raises(ValueError):
        _lib.check(L.klc_mxfp4_dequant(None, None, -1, 3, None, 0, None))


@pytest.mark.parametrize("path", ["simt", "tc", "auto"])
def test_workspace_size_grows_with_tokens(path):
    L = _lib.lib()
    sizes = []
    for T in (1, 8, 256, 4096):
        d = _lib.KlcDims(T, 2880, 2880, 128, 4, _lib.PATH_CODE[path])
        n = ctypes.c_size_t(0)
        _lib.check(L.klc_moe_workspace_size(ctypes.byref(d), ctypes.byref(n)))
        sizes.append(n.value)
    assert sizes == sorted(sizes) and sizes[0] > 0
    # the permuted activations, intermediate and expert outputs dominate: ~T*k rows
    assert sizes[-1] > 4096 * 4 * 2880 * 2 * 3


def test_workspace_rejects_bad_dims():
    L = _lib.lib()
    n = ctypes.c_size_t(0)
    for d in (
        _lib.KlcDims(8, 2880, 2880, 128, 9, 0),   # k > 8
        _lib.KlcDims(8, 2881, 2880, 128, 4, 0),   # hidden not a multiple of 64
        _lib.KlcDims(8, 2880, 2880, 0, 4, 0),     # no experts
        _lib.KlcDims(-1, 2880, 2880, 128, 4, 0),  # negative tokens
        _lib.KlcDims(8, 2880, 2880, 128, 4, 5),   # unknown path
    ):
        assert L.klc_moe_workspace_size(ctypes.byref(d), ctypes.byref(n)) == _lib.KLC_ERR_INVALID


def test_experts_reject_small_workspace():
    L = _lib.lib()
    d = _lib.KlcDims(8, 128, 128, 8, 2, 1)
    w = _lib.KlcWeights(16, 16, 16, 16, 16, 16, 16, 16, 7.0, 1.702)
    st = L.klc_moe_experts(ctypes.byref(d), ctypes.byref(w), 16, 16, 16, 0, 16, None, None, 256, 64, None)
    assert st == _lib.KLC_ERR_WORKSPACE


def test_workspace_growth_keeps_replaced_buffers(monkeypatch):
    """A larger call replaces the workspace of its (device, stream) but keeps the
    old one allocated (a CUDA graph captured with it still writes there on
    replay); another stream gets a workspace of its own."""
    import torch

    from kcapw_klcquant_b200 import moe

    real_empty = torch.empty
    monkeypatch.setattr(moe.torch, "empty", lambda n, dtype=None, device=None: real_empty(n, dtype=dtype))
    monkeypatch.setattr(moe, "_WORKSPACES", {})
    monkeypatch.setattr(moe, "_RETIRED_WORKSPACES", [])
    dev = torch.device("cuda", 0)
    a = moe.workspace(dev, 1000, stream=0)
    assert a.numel() >= 1 << 20  # at least 1 MiB
    assert moe.workspace(dev, 5000, stream=0) is a  # reused while large enough
    other = moe.workspace(dev, 1000, stream=0x1234)
    assert other is not a  # a second stream never shares scratch with the first
    b = moe.workspace(dev, (1 << 20) + 1, stream=0)
    assert b is not a and b.numel() >= (1 << 20) + 1
    assert moe._RETIRED_WORKSPACES == [a]
    assert moe.workspace(dev, 10, stream=0) is b
    assert moe.workspace(dev, 10, stream=0x1234) is other


def test_noalloc_validates_like_the_workspace_entry_point():
    """klc_moe_experts_noalloc runs the same host checks as klc_moe_experts before
    any size arithmetic or launch: misaligned expert blocks, an unbounded token
    count and bad shapes come back as KLC_ERR_INVALID (no GPU is touched)."""
    L = _lib.lib()
    d = _lib.KlcDims(8, 2880, 2880, 32, 4, _lib.KLC_PATH_SIMT)
    good = _lib.KlcWeights(256, 256, 256, 256, 256, 256, 256, 256, 7.0, 1.702)
    for field in ("gu_blocks", "dn_blocks"):
        w = _lib.KlcWeights(256, 256, 256, 256, 256, 256, 256, 256, 7.0, 1.702)
        setattr(w, field, 256 + 8)  # 8-byte aligned only: the 128-bit weight loads would fault
        st, msg = _status_and_msg(L.klc_moe_experts_noalloc(ctypes.byref(d), ctypes.byref(w), 256, 256, 256,
                                                            _lib.KLC_PREC_BF16, 256, None, None, None))
        assert st == _lib.KLC_ERR_INVALID and "aligned" in msg, (field, msg)
    huge = _lib.KlcDims(1 << 40, 2880, 2880, 32, 4, _lib.KLC_PATH_SIMT)
    st, msg = _status_and_msg(L.klc_moe_experts_noalloc(ctypes.byref(huge), ctypes.byref(good), 256, 256, 256,
                                                        _lib.KLC_PREC_BF16, 256, None, None, None))
    assert st == _lib.KLC_ERR_INVALID and "tokens" in msg
    bad = _lib.KlcDims(8, 2881, 2880, 32, 4, _lib.KLC_PATH_SIMT)
    st, _ = _status_and_msg(L.klc_moe_experts_noalloc(ctypes.byref(bad), ctypes.byref(good), 256, 256, 256,
                                                      _lib.KLC_PREC_BF16, 256, None, None, None))
    assert st == _lib.KLC_ERR_INVALID
