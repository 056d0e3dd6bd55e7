"""Fused Q/K RMSNorm, RoPE and K/V packing for attention.

Mirrors src/qwen_image_accel/kernels/attention.py (prepare_attention_inputs)
and adds joint_qk_norm_rope for the dual-stream (v1) joint [text, image]
sequence.
"""
from __future__ import annotations

import torch

from .. import _lib


def prepare_attention_inputs(q, k, v, norm_q, norm_k, freqs, cached_k, cached_v):
    """Return fused Q/K/V, or None when the original operators should be used."""
    if (q.ndim != 4 or q.shape[-1] != 128 or q.shape[1] == 0 or k.shape != q.shape or v.shape != q.shape
            or freqs is None or freqs.dtype != torch.complex64 or freqs.shape != (q.shape[1], 64)
            or not freqs.is_contiguous() or freqs.device != q.device
            or cached_k.ndim != 4 or cached_k.shape[0] != q.shape[0] or cached_k.shape[2:] != q.shape[2:]
            or cached_v.shape != cached_k.shape):
        return None
    for t in (q, k, v, cached_k, cached_v):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.device != q.device or not t.is_contiguous():
            return None
    for norm in (norm_q, norm_k):
        if (norm.weight is None or getattr(norm, "bias", None) is not None or norm.weight.shape != (128,)
                or norm.weight.dtype != torch.bfloat16 or norm.weight.device != q.device
                or not norm.weight.is_contiguous()):
            return None
    b, s, h, d = q.shape
    p = cached_k.shape[1]
    oq = torch.empty_like(q)
    ok = torch.empty((b, s + p, h, d), device=q.device, dtype=q.dtype)
    ov = torch.empty_like(ok)
    _lib.call("qia_qknorm_rope_pack", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v),
              _lib.ptr(cached_k) if p else None, _lib.ptr(cached_v) if p else None,
              _lib.ptr(norm_q.weight), _lib.ptr(norm_k.weight), _lib.ptr(torch.view_as_real(freqs)),
              _lib.ptr(oq), _lib.ptr(ok), _lib.ptr(ov), b, s, p, h, d, float(norm_q.eps), float(norm_k.eps),
              _lib.stream(q.device))
    return oq, ok, ov


def joint_qk_norm_rope(qkv: torch.Tensor, weight_q: torch.Tensor, weight_k: torch.Tensor, freqs: torch.Tensor,
                       out_q: torch.Tensor, out_k: torch.Tensor, out_v: torch.Tensor, seq_offset: int,
                       eps: float = 1e-6) -> None:
    """Normalise + rotate one stream's q|k|v projection (B, L, 3*H*128) into
    rows [seq_offset, seq_offset + L) of the joint (B, S, H, 128) outputs.

    freqs: float32 (L, 64, 2) (complex64 viewed as real) for this segment."""
    _lib.require_cuda(qkv, weight_q, weight_k, freqs, out_q, out_k, out_v)
    b, seg, cols = qkv.shape
    _, total, h, d = out_q.shape
    if qkv.stride(-1) != 1 or qkv.stride(0) != seg * qkv.stride(1):
        raise NotImplementedError("joint_qk_norm_rope: qkv rows must be evenly strided")
    _lib.call("qia_qknorm_rope_segment", _lib.ptr(qkv), qkv.stride(1), _lib.ptr(weight_q), _lib.ptr(weight_k),
              _lib.ptr(freqs), _lib.ptr(out_q), _lib.ptr(out_k), _lib.ptr(out_v), b, seg, seq_offset, total, h, d,
              float(eps), float(eps), _lib.stream(qkv.device))
