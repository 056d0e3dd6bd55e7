"""BF16 gated residual and rotary embedding.

Mirrors src/qwen_image_accel/kernels/elementwise.py (residual, rope_qk).
"""
from __future__ import annotations

import torch

from .. import _lib


def residual(h: torch.Tensor, x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """h + bf16(x * gate); gate is (B, 1, D) broadcast over the sequence."""
    _lib.require_cuda(h, x, gate)
    if (h.dtype != torch.bfloat16 or x.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16
            or not h.is_contiguous() or not x.is_contiguous() or x.shape != h.shape or h.ndim != 3
            or gate.shape not in ((h.shape[0], 1, h.shape[-1]), (1, 1, h.shape[-1])) or not gate.is_contiguous()):
        raise NotImplementedError("residual: expects contiguous bf16 (B, S, D) h/x and (B, 1, D) or (1, 1, D) gate")
    out = torch.empty_like(h)
    b, s, d = h.shape
    rows_per_gate = s if gate.shape[0] == b else b * s
    _lib.call("qia_gated_residual", _lib.ptr(h), _lib.ptr(x), _lib.ptr(gate), _lib.ptr(out), b * s, d, rows_per_gate,
              _lib.stream(h.device))
    return out


def rope_qk(q: torch.Tensor, k: torch.Tensor, freqs: torch.Tensor):
    """Complex RoPE on interleaved pairs; freqs complex64 (S, D/2)."""
    _lib.require_cuda(q, k, freqs)
    if (q.ndim != 4 or q.shape != k.shape or q.shape[-1] != 128 or q.dtype != torch.bfloat16
            or k.dtype != torch.bfloat16 or not q.is_contiguous() or not k.is_contiguous()
            or freqs.dtype != torch.complex64 or freqs.shape != (q.shape[1], 64) or not freqs.is_contiguous()):
        raise NotImplementedError("rope_qk: expects contiguous bf16 (B, S, H, 128) and complex64 (S, 64) freqs")
    out_q, out_k = torch.empty_like(q), torch.empty_like(k)
    b, s, h, d = q.shape
    _lib.call("qia_rope_qk", _lib.ptr(q), _lib.ptr(k), _lib.ptr(torch.view_as_real(freqs)), _lib.ptr(out_q),
              _lib.ptr(out_k), b, s, h, d, _lib.stream(q.device))
    return out_q, out_k
