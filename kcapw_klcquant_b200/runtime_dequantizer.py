"""Drop-in ``RuntimeDequantizer`` with device kernels (klcquant runtime_dequantizer.py:1-59).

Same ``QuantizedTensorMeta``, ``parse_bool`` and ``dequantize(meta, data,
scale, device, dtype)`` signature.  The reference unpacks q1-q4 artefacts on
the CPU and then scales on the target device; here the packed bytes are
copied once to the device and ``klc_runtime_dequant`` unpacks, scales and
rounds in one pass.  Errors match the reference: ``ValueError`` when a
quantized tensor has no scale or a pruned tensor has no index tensor.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

QUANT_MODES = ("fp16", "q16", "q8", "q4", "q3", "q2", "q1", "pruned")


@dataclass(frozen=True)
class QuantizedTensorMeta:
    name: str
    mode: str
    shape: tuple[int, ...]
    dtype: str
    bits: int
    packed: bool
    group: str
    file: str


def parse_bool(value: str | bool | None) -> bool:
    if isinstance(value, bool):
        return value
    return str(value).strip().lower() in {"1", "true", "yes", "on"}


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


class RuntimeDequantizer:
    def dequantize(self, meta: QuantizedTensorMeta, data: torch.Tensor, scale: torch.Tensor | None, device: torch.device,
                   dtype: torch.dtype = torch.float16) -> torch.Tensor:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("RuntimeDequantizer runs on CUDA devices only")
        if dtype not in _lib.DTYPE_CODE:
            raise ValueError(f"unsupported dtype {dtype}")
        numel = _numel(meta.shape)
        out = torch.empty(numel, dtype=dtype, device=device)
        L = _lib.lib()
        if meta.mode == "fp16":
            src = data.to(device=device, non_blocking=True).contiguous()
            if src.dtype not in _lib.DTYPE_CODE:
                src = src.float()
            with torch.cuda.device(device):
                _lib.check(L.klc_runtime_dequant(0, src.data_ptr(), _lib.DTYPE_CODE[src.dtype], None, None, 0, 16, numel,
                                                 out.data_ptr(), _lib.DTYPE_CODE[dtype], _lib.stream_ptr()))
            return out.reshape(meta.shape)
        if meta.mode == "pruned":
            if scale is None:
                raise ValueError(f"{meta.name} is pruned but has no sparse index tensor")
            vals = data.to(device=device, non_blocking=True).contiguous()
            if vals.dtype not in _lib.DTYPE_CODE:
                vals = vals.float()
            index = scale.to(device=device, dtype=torch.int64).contiguous()
            with torch.cuda.device(device):
                _lib.check(L.klc_runtime_dequant(3, vals.data_ptr(), _lib.DTYPE_CODE[vals.dtype], None, index.data_ptr(), index.numel(),
                                                 16, numel, out.data_ptr(), _lib.DTYPE_CODE[dtype], _lib.stream_ptr()))
            return out.reshape(meta.shape)
        if scale is None:
            raise ValueError(f"{meta.name} is quantized but has no scale tensor")
        s = scale.to(device=device, dtype=torch.float32).reshape(-1).contiguous()
        if meta.packed:
            src = data.to(device=device, non_blocking=True).contiguous().view(torch.uint8)
            mode, bits = 1, int(meta.bits)
        else:
            src = data.to(device=device, non_blocking=True).contiguous()
            if src.dtype == torch.int8:
                bits = 8
            elif src.dtype == torch.int16:
                bits = 16
            else:
                raise ValueError(f"unpacked quantized data must be int8 or int16, got {src.dtype}")
            mode = 2
        with torch.cuda.device(device):
            _lib.check(L.klc_runtime_dequant(mode, src.data_ptr(), 0, s.data_ptr(), None, src.numel(), bits, numel, out.data_ptr(),
                                             _lib.DTYPE_CODE[dtype], _lib.stream_ptr()))
        return out.reshape(meta.shape)
