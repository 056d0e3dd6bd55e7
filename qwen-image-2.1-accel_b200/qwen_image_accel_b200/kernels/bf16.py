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


def install_swiglu(transformer):
    for block in transformer.transformer_blocks:
        def forward(self, hidden_states):
            return self.out(swiglu(self.gate_layer(hidden_states), self.proj(hidden_states)))
        block.img_mlp.forward = types.MethodType(forward, block.img_mlp)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    _lib.require_cuda(x, weight)
    if (x.dtype != torch.bfloat16 or not x.is_contiguous() or x.shape[-1] != 128
            or weight.dtype != torch.bfloat16 or weight.shape != (128,) or not weight.is_contiguous()):
        raise NotImplementedError("rms_norm: expects contiguous bf16 (..., 128) and a bf16 (128,) weight")
    out = torch.empty_like(x)
    _lib.call("qia_rms_norm", _lib.ptr(x), _lib.ptr(weight), _lib.ptr(out), x.numel() // 128, 128, float(eps),
              _lib.stream(x.device))
    return out


def install_qk_norm(transformer):
    for block in transformer.transformer_blocks:
        for norm in (block.attn.norm_q, block.attn.norm_k):
            eager = norm.forward

            def forward(self, x, _eager=eager):
                if (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous()
                        and x.shape[-1] == 128 and self.weight is not None
                        and self.weight.dtype == torch.bfloat16 and self.weight.is_contiguous()
                        and self.bias is None):
                    return rms_norm(x, self.weight, self.eps)
                return _eager(x)
            norm.forward = types.MethodType(forward, norm)
