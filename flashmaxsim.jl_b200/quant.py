"""Per-token symmetric INT8 index (quant.jl:1-49)."""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .errors import ArgumentError, DimensionMismatch


@dataclass(frozen=True)
class Int8Index:
    """INT8 token codes plus per-token absmax scales (quant.jl:11-14).

    codes: (..., T, dim) int8 (Julia (dim, T, ...)); scales: (..., T)."""
    codes: torch.Tensor
    scales: torch.Tensor

    def __repr__(self):
        return (f"Int8Index(codes={tuple(self.codes.shape)}, scales={tuple(self.scales.shape)}, "
                f"eltype={self.scales.dtype})")

    def to(self, device):
        return Int8Index(self.codes.to(device), self.scales.to(device))


def require_int8_index(d: Int8Index):
    """require_int8_index (quant.jl:142-153)."""
    if d.codes.shape[:-1] != d.scales.shape:
        raise DimensionMismatch("Int8Index token count")


def quantize_int8_symmetric(x: torch.Tensor) -> Int8Index:
    """quantize_int8_symmetric (quant.jl:42-49) on the GPU: per-token
    scale = max(max(absmax, T(1f-8))/T(127), floatmin(T)), codes =
    round(clamp(x/scale, -127, 127)) with ties to even, every op in T."""
    if x.device.type != "cuda":
        raise ArgumentError("quantize_int8_symmetric runs on CUDA tensors only")
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ArgumentError(f"quantize_int8_symmetric: unsupported dtype {x.dtype}")
    x = x.contiguous()
    dim = x.shape[-1]
    ntok = x.numel() // dim if dim > 0 else int(torch.tensor(x.shape[:-1]).prod().item())
    codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scales = torch.empty(x.shape[:-1], dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("fms_quantize_int8", _lib.DTYPE_CODE[x.dtype], _lib.ptr(x), dim, ntok,
                  _lib.ptr(codes), _lib.ptr(scales), _lib.stream_of(x.device))
    return Int8Index(codes, scales)


def dequant_int8(idx: Int8Index) -> torch.Tensor:
    """dequant_int8 (quant.jl:56-58): T.(codes) .* scales."""
    return idx.codes.to(idx.scales.dtype) * idx.scales.unsqueeze(-1)
