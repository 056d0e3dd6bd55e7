"""LayerNorm + timestep scale (+ shift) in PyTorch's CUDA LayerNorm reduction order.

Mirrors src/qwen_image_accel/kernels/layernorm.py (layer_norm_scale), extended
with the optional shift of the dual-stream (v1) AdaLN and any width that is a
multiple of 512 (3072 and 4096 included).
"""
from __future__ import annotations

import torch

from .. import _lib


def _check(x, scale, shift, norm):
    _lib.require_cuda(x, scale, shift)
    if getattr(norm, "elementwise_affine", False):
        raise NotImplementedError("affine LayerNorm is not on the fused path; use norm(x) * scale")
    d = x.shape[-1]
    if (x.ndim != 3 or x.dtype != torch.bfloat16 or not x.is_contiguous() or d % 512 or d > 8192
            or x.numel() == 0 or tuple(norm.normalized_shape) != (d,)):
        raise NotImplementedError(f"layer_norm_scale: unsupported input {tuple(x.shape)} {x.dtype}")
    for v in (scale, shift):
        if v is not None and (v.shape not in ((x.shape[0], 1, d), (1, 1, d)) or v.dtype != torch.bfloat16
                              or not v.is_contiguous() or v.shape[0] != scale.shape[0]):
            raise NotImplementedError("layer_norm_scale: scale/shift must be contiguous bf16 (B, 1, D) or (1, 1, D)")


def layer_norm_scale(x: torch.Tensor, scale: torch.Tensor, norm, shift: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(LN(x)) * scale [+ shift], each product/sum rounded to bf16.

    ``scale`` is the precomputed ``1 + s`` vector, as in the reference; a
    (1, 1, D) scale/shift is shared by every batch row."""
    _check(x, scale, shift, norm)
    out = torch.empty_like(x)
    b, s, d = x.shape
    rows_per_vector = s if scale.shape[0] == b else b * s
    _lib.call("qia_ln_mod", _lib.ptr(x), _lib.ptr(scale), _lib.ptr(shift), _lib.ptr(out), b * s, d, rows_per_vector,
              float(norm.eps), _lib.stream(x.device))
    return out
