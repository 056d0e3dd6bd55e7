"""AdaLN modulation vectors of the dual-stream block (qia_adaln_modulation).

The v1 block computes its six per-stream modulation chunks (shift1, scale1,
gate1, shift2, scale2, gate2) with img_mod / txt_mod = Linear(SiLU(temb)) and
uses 1 + scale (WHL:diffusers/models/transformers/transformer_qwenimage.py:
683-717). One launch computes a block's 12 chunks from its stacked weights,
returning the scale chunks as 1 + scale.
"""
from __future__ import annotations

import torch

from .. import _lib


def adaln_modulation(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, unit: int,
                     out: torch.Tensor | None = None, ctas: int | None = None) -> torch.Tensor:
    """x: SiLU(temb) [k] or [1, k] bf16; weight [n, k], bias [n] bf16 with n a
    multiple of 6 * unit; returns [n] bf16 with chunks 1 and 4 of every six as
    1 + scale. ctas bounds the grid (default: 8 per SM)."""
    _lib.require_cuda(x, weight, bias)
    n, k = weight.shape
    if x.numel() != k or x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or bias.dtype != torch.bfloat16:
        raise NotImplementedError("adaln_modulation: bf16 x [k], weight [n, k], bias [n]")
    if not (x.is_contiguous() and weight.is_contiguous() and bias.is_contiguous()):
        raise NotImplementedError("adaln_modulation: contiguous inputs")
    if out is None:
        out = torch.empty(n, device=weight.device, dtype=torch.bfloat16)
    if ctas is None:
        ctas = 8 * torch.cuda.get_device_properties(weight.device).multi_processor_count
    _lib.call("qia_adaln_modulation", _lib.ptr(x), _lib.ptr(weight), _lib.ptr(bias), _lib.ptr(out), n, k, unit,
              ctas, _lib.stream(weight.device))
    return out
