"""Block-scaled E4M3 quantization and the NVIDIA 128x4 scale layout.

Mirrors src/qwen_image_accel/kernels/mxfp8.py (Quantized, padded_rows, quantize).
"""
from __future__ import annotations

from typing import NamedTuple

import torch

from .. import _lib


class Quantized(NamedTuple):
    """An MXFP8 activation: padded E4M3 values plus their swizzled E8M0 scales."""

    values: torch.Tensor     # (rows padded to 128, K) float8_e4m3fn
    scales: torch.Tensor     # flat float8_e8m0fnu in the 128x4 blocked order
    rows: int                # live rows, before padding
    shape: torch.Size        # logical shape of the tensor this came from


def padded_rows(rows: int) -> int:
    """MXFP8 scales are tiled over 128 rows, so M is padded to a multiple of 128."""
    return (rows + 127) // 128 * 128


def empty_quantized(rows: int, k: int, device, shape=None) -> Quantized:
    padded = padded_rows(rows)
    values = torch.empty((padded, k), device=device, dtype=torch.float8_e4m3fn)
    scales = torch.empty(padded * k // 32, device=device, dtype=torch.uint8)
    return Quantized(values, scales.view(torch.float8_e8m0fnu), rows,
                     torch.Size(shape) if shape is not None else torch.Size((rows, k)))


def quantize(x: torch.Tensor) -> Quantized:
    """Quantize a BF16 ``(M, K)`` activation (unit column stride) to MXFP8."""
    _lib.require_cuda(x)
    if x.ndim != 2 or x.dtype != torch.bfloat16 or x.stride(1) != 1:
        raise ValueError("quantize expects a bf16 (M, K) tensor with unit column stride")
    m, k = x.shape
    out = empty_quantized(m, k, x.device, x.shape)
    _lib.call("qia_mxfp8_quantize", _lib.ptr(x), x.stride(0), _lib.ptr(out.values), _lib.ptr(out.scales),
              m, k, _lib.stream(x.device))
    return out
