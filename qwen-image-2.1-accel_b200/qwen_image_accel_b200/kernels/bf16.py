"""BF16 pointwise fusion with explicit rounding: SwiGLU, GELU-tanh, per-head RMSNorm.

Mirrors src/qwen_image_accel/kernels/bf16.py (swiglu, install_swiglu,
rms_norm, install_qk_norm) and adds the v1 FeedForward's GELU-tanh.
"""
from __future__ import annotations

import types

import torch

from .. import _lib


def swiglu(gate: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(gate, value)
    if (gate.dtype != torch.bfloat16 or value.dtype != torch.bfloat16 or gate.shape != value.shape
            or not gate.is_contiguous() or not value.is_contiguous() or gate.numel() % 8):
        raise NotImplementedError("swiglu: expects contiguous bf16 tensors of equal shape")
    out = torch.empty_like(gate)
    _lib.call("qia_swiglu", _lib.ptr(gate), _lib.ptr(value), _lib.ptr(out), gate.numel(), _lib.stream(gate.device))
    return out


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.numel() % 8:
        raise NotImplementedError("gelu_tanh: expects a contiguous bf16 tensor")
    out = torch.empty_like(x)
    _lib.call("qia_gelu_tanh", _lib.ptr(x), _lib.ptr(out), x.numel(), _lib.stream(x.device))
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    _lib.require_cuda(x, weight)
    if (x.dtype != torch.bfloat16 or not x.is_contiguous() or x.shape[-1] != 128
            or weight.dtype != torch.bfloat16 or weight.shape != (128,) or not weight.is_contiguous()):
        raise NotImplementedError("rms_norm: expects contiguous bf16 (..., 128) and a bf16 (128,) weight")
    out = torch.empty_like(x)
    _lib.call("qia_rms_norm", _lib.ptr(x), _lib.ptr(weight), _lib.ptr(out), x.numel() // 128, 128, float(eps),
              _lib.stream(x.device))
    return out


def _qk_norm_kernel_ok(norm, x) -> bool:
    """An input the qia_rms_norm kernel takes: contiguous CUDA bf16 rows of 128
    and a bf16 weight without bias."""
    w = getattr(norm, "weight", None)
    return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[-1] == 128
            and w is not None and w.dtype == torch.bfloat16 and w.is_contiguous()
            and getattr(norm, "bias", None) is None)


def install_qk_norm(transformer) -> None:
    """Give every block's per-head Q/K RMSNorm (attn.norm_q / attn.norm_k) the
    qia_rms_norm kernel (Diffusers RMSNorm's two roundings) for the inputs it
    takes; other inputs keep the module's own forward (the reference's
    install_qk_norm contract, src/qwen_image_accel/kernels/bf16.py:66-77)."""
    for block in transformer.transformer_blocks:
        for norm in (block.attn.norm_q, block.attn.norm_k):
            native = norm.forward
            norm.forward = types.MethodType(
                lambda mod, x, _native=native: rms_norm(x, mod.weight, mod.eps) if _qk_norm_kernel_ok(mod, x)
                else _native(x), norm)


def install_swiglu(transformer) -> None:
    """Give every block's SwiGLU MLP (img_mlp: gate_layer, proj, out) the
    qia_swiglu kernel between its projections (the reference's install_swiglu
    contract, src/qwen_image_accel/kernels/bf16.py:39-43). Blocks whose decode
    is routed (optimizations/decode.py) already run this MLP and are left
    alone."""
    routed = getattr(transformer, "_qia_decode", None)
    for block in transformer.transformer_blocks:
        if routed is not None:
            continue
        block.img_mlp.forward = types.MethodType(
            lambda mlp, x: mlp.out(swiglu(mlp.gate_layer(x).contiguous(), mlp.proj(x).contiguous())), block.img_mlp)
