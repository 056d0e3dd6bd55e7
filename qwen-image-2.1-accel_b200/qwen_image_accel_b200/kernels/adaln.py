"""The AdaLN + gated-residual composite of the dual-stream block, in one pass.

out = r + gate * (LN(x) * (1 + scale) + shift), every eager bf16 op boundary
kept as a rounding point (WHL:diffusers/models/transformers/
transformer_qwenimage.py:741-767, composed).
"""
from __future__ import annotations

import torch

from .. import _lib


def adaln_residual(x: torch.Tensor, r: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                   gate: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x, r: (B, S, D) bf16; scale (= 1 + s), shift, gate: (B, 1, D) bf16."""
    _lib.require_cuda(x, r, scale, shift, gate)
    b, s, d = x.shape
    for t in (x, r):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape != (b, s, d):
            raise NotImplementedError("adaln_residual: x and r must be contiguous bf16 (B, S, D)")
    for t in (scale, shift, gate):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape != (b, 1, d):
            raise NotImplementedError("adaln_residual: scale/shift/gate must be contiguous bf16 (B, 1, D)")
    out = torch.empty_like(x)
    _lib.call("qia_adaln_residual", _lib.ptr(x), _lib.ptr(r), _lib.ptr(scale), _lib.ptr(shift), _lib.ptr(gate),
              _lib.ptr(out), b * s, d, s, float(eps), _lib.stream(x.device))
    return out
