"""Fused MXFP8 epilogues: LayerNorm/SwiGLU results quantized in the same pass.

Mirrors src/qwen_image_accel/kernels/epilogue.py (layer_norm_scale_quantize,
swiglu_quantize): each returns a Quantized, or None when the input is outside
the fused path (the reference's contract).
"""
from __future__ import annotations

import torch

from .. import _lib
from .mxfp8 import Quantized, empty_quantized


def layer_norm_scale_quantize(x: torch.Tensor, scale: torch.Tensor, norm,
                              shift: torch.Tensor | None = None) -> Quantized | None:
    """LayerNorm, timestep scale (+ shift) and MXFP8 quantization in one pass, or None."""
    _lib.require_cuda(x, scale, shift)
    d = x.shape[-1] if x.ndim else 0
    if (x.ndim != 3 or x.dtype != torch.bfloat16 or not x.is_contiguous() or d % 512 or d > 8192
            or x.numel() == 0 or getattr(norm, "elementwise_affine", False)
            or tuple(norm.normalized_shape) != (d,)):
        return None
    for v in (scale, shift):
        if v is not None and (v.shape not in ((x.shape[0], 1, d), (1, 1, d)) or v.dtype != torch.bfloat16
                              or not v.is_contiguous() or v.shape[0] != scale.shape[0]):
            return None
    b, s, _ = x.shape
    rows_per_vector = s if scale.shape[0] == b else b * s
    out = empty_quantized(b * s, d, x.device, x.shape)
    _lib.call("qia_ln_mod_quant", _lib.ptr(x), _lib.ptr(scale), _lib.ptr(shift), _lib.ptr(out.values),
              _lib.ptr(out.scales), b * s, d, rows_per_vector, float(norm.eps), _lib.stream(x.device))
    return out


def layer_norm_scale_quantize_grouped(items, norm) -> list:
    """layer_norm_scale_quantize of one or two (x, scale, shift) inputs with the
    same D (the block's image and text streams) in one launch; each result
    equals the single call's. Raises where the single call would return None."""
    import ctypes
    probs = (_lib.LnProblem * len(items))()
    outs = []
    d = items[0][0].shape[-1]
    for slot, (x, scale, shift) in zip(probs, items):
        _lib.require_cuda(x, scale, shift)
        if (x.ndim != 3 or x.dtype != torch.bfloat16 or not x.is_contiguous() or x.shape[-1] != d or d % 512
                or d > 8192 or x.numel() == 0 or getattr(norm, "elementwise_affine", False)
                or tuple(norm.normalized_shape) != (d,)):
            raise NotImplementedError("grouped LayerNorm: contiguous bf16 (B, S, D), D % 512 == 0, no affine")
        for v in (scale, shift):
            if v is not None and (v.shape not in ((x.shape[0], 1, d), (1, 1, d)) or v.dtype != torch.bfloat16
                                  or not v.is_contiguous() or v.shape[0] != scale.shape[0]):
                raise NotImplementedError("grouped LayerNorm: scale/shift must be (B or 1, 1, D) bf16")
        b, s_, _ = x.shape
        out = empty_quantized(b * s_, d, x.device, x.shape)
        outs.append(out)
        slot.x, slot.scale, slot.shift = _lib.ptr(x), _lib.ptr(scale), _lib.ptr(shift)
        slot.q_values, slot.q_scales = _lib.ptr(out.values), _lib.ptr(out.scales)
        slot.rows, slot.rows_per_batch = b * s_, (s_ if scale.shape[0] == b else b * s_)
    _lib.call("qia_ln_mod_quant_grouped", ctypes.addressof(probs), len(items), d, float(norm.eps),
              _lib.stream(items[0][0].device))
    return outs


def swiglu_quantize(gate: torch.Tensor, value: torch.Tensor) -> Quantized | None:
    """SwiGLU and MXFP8 quantization in one pass, or None when unsupported."""
    _lib.require_cuda(gate, value)
    if (gate.dtype != torch.bfloat16 or value.dtype != torch.bfloat16 or gate.shape != value.shape
            or not gate.is_contiguous() or not value.is_contiguous() or gate.ndim != 2
            or gate.shape[-1] % 128 or gate.numel() == 0):
        return None
    rows, width = gate.shape
    out = empty_quantized(rows, width, gate.device, gate.shape)
    _lib.call("qia_swiglu_quant", _lib.ptr(gate), _lib.ptr(value), _lib.ptr(out.values), _lib.ptr(out.scales),
              rows, width, _lib.stream(gate.device))
    return out
